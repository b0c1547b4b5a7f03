/*
 * warp_route_b200.h — C ABI of the B200-native fused decode-time MoE layer.
 *
 * Plain pointers and sizes only: no torch, no C++ types.  Every entry point
 * returns a wr_status_t and never calls exit(); every launch goes on the
 * stream the caller passes, and no entry point blocks the host or allocates
 * device memory unless its comment says so.  The caller owns every buffer.
 *
 * Each declaration names the warp-route interface it replaces, as
 * path:line within the warp-route project (anishesg/warp-route).
 *
 * Arithmetic contract (shared by all compute entry points; follows
 * src/fused_moe.cu:100-226 and tests/test_python.py:15-37):
 *   logits[e] = gate_w[e,:] . x   (+ router_bias[e] when given), fp32;
 *   probs     = softmax(logits) over all E experts, fp32;
 *   top-K     = iterative argmax over the logits with strict '>', so ties go
 *               to the lowest expert index; weight_k = probs[id_k] (NOT
 *               renormalised over the K selected experts);
 *   out       = sum_k weight_k * Wd_k (silu(Wg_k x) * (Wu_k x)),
 *               silu(g) = g / (1 + exp(-g)); accumulated and returned in fp32.
 * The logits are computed in fp32 with one fixed reduction order (the row's
 * 16-byte vectors cut into 8 segments; per segment a 32-lane strided fma
 * sweep and a 16/8/4/2/1 xor tree; segment sums added left to right), so the
 * selected expert indices are reproducible bit for bit on any device and by
 * the CPU oracle.
 */
#ifndef WARP_ROUTE_B200_H
#define WARP_ROUTE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WR_API __attribute__((visibility("default")))
#else
#define WR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque stream handle: a cudaStream_t passed through unchanged (NULL = the
 * legacy default stream, as in the warp-route launchers). */
typedef void* wr_stream_t;

typedef enum wr_status {
  WR_OK = 0,
  WR_ERR_INVALID = 1,      /* bad argument: null pointer, shape, top_k, ... */
  WR_ERR_UNSUPPORTED = 2,  /* valid in warp-route but outside this build's limits */
  WR_ERR_CUDA = 3,         /* a CUDA runtime call failed (see wr_last_error_string) */
  WR_ERR_TIMEOUT = 4,      /* a bounded device-side wait gave up */
  WR_ERR_WORKSPACE = 5,    /* workspace missing, misaligned or too small */
  WR_ERR_TOO_SMALL = 6,    /* weight_buf smaller than the layout requires */
  WR_ERR_COMM = 7          /* multi-GPU communicator error */
} wr_status_t;

typedef enum wr_dtype {
  WR_DTYPE_F32 = 0,   /* float32 x / gate_w / weight_buf (warp-route's only dtype) */
  WR_DTYPE_BF16 = 1   /* bfloat16 x / gate_w / weight_buf, fp32 accumulation and output */
} wr_dtype_t;

/* Shape of one MoE layer.  Replaces ExpertLayoutConfig + top_k
 * (src/expert_layout.cuh:20-24, src/fused_moe.cuh:17-22).
 * ep_first_expert / ep_num_local describe an expert-parallel shard: the
 * weight_buf then holds experts [ep_first_expert, ep_first_expert +
 * ep_num_local) packed from slot 0, the router still scores all num_experts
 * experts, and selected experts outside the shard contribute zero.
 * ep_num_local = 0 means every expert is local (no expert parallelism). */
typedef struct wr_moe_desc {
  int32_t num_experts;
  int32_t hidden_dim;
  int32_t intermediate_dim;
  int32_t top_k;
  int32_t dtype;            /* wr_dtype_t */
  int32_t ep_first_expert;
  int32_t ep_num_local;
  int32_t reserved;
  const float* router_bias; /* optional fp32 [num_experts] added to the logits; NULL = none */
} wr_moe_desc_t;

/* Byte offsets inside one packed expert block.  Replaces ExpertOffsets
 * (src/expert_layout.cuh:27-32). */
typedef struct wr_expert_offsets {
  int64_t gate_proj_offset;
  int64_t up_proj_offset;
  int64_t down_proj_offset;
  int64_t expert_stride;    /* 128-byte aligned */
} wr_expert_offsets_t;

/* ---- layout ------------------------------------------------------------ */

/* Per-expert [gate I x H | up I x H | down H x I] row-major offsets for an
 * element size of elt_bytes (4 reproduces warp-route's float layout byte for
 * byte).  Replaces compute_offsets (src/expert_layout.cuh:34-47). */
WR_API wr_status_t wr_expert_offsets(int32_t hidden_dim, int32_t intermediate_dim,
                              int32_t elt_bytes, wr_expert_offsets_t* out);

/* Bytes of a packed buffer of num_experts experts.  Replaces
 * total_weight_bytes (src/expert_layout.cuh:74-77). */
WR_API int64_t wr_total_weight_bytes(int32_t num_experts, int32_t hidden_dim,
                              int32_t intermediate_dim, int32_t elt_bytes);

/* ---- status ------------------------------------------------------------ */

WR_API const char* wr_status_string(wr_status_t s);
/* Text of the most recent error raised on the calling thread (argument
 * checks name the argument, as the TORCH_CHECK messages of
 * src/bindings.cpp:9-23,40-43,75-83 do). */
WR_API const char* wr_last_error_string(void);
/* Library version string. */
WR_API const char* wr_version(void);

/* ---- router ------------------------------------------------------------ */

/* Router + softmax + top-K for num_tokens tokens (x: [num_tokens, H]).
 * Writes fp32 logits [T,E] (optional, may be NULL), int32 ids [T,K] and fp32
 * weights [T,K].  Replaces warp_gate_topk (src/gate.cu:103-116, declared
 * src/gate.cuh:24-30) and the inlined router of src/fused_moe.cu:100-150. */
WR_API wr_status_t wr_router_topk(const wr_moe_desc_t* desc, int32_t num_tokens,
                           const void* x, const void* gate_w,
                           float* logits_out, int32_t* topk_ids,
                           float* topk_weights, wr_stream_t stream);

/* ---- fused layer, one token ------------------------------------------- */

/* Device workspace the fused single-token and batched entry points need for
 * num_tokens tokens (bytes, 256-byte aligned base required).  The workspace
 * must be zero-filled before its first use; every call leaves it reusable.
 * Calls that share one workspace must not overlap on the GPU. */
WR_API size_t wr_fused_moe_workspace_size(const wr_moe_desc_t* desc, int32_t num_tokens);

/* One decode token: x [H] -> out [H] (fp32).  topk_ids [K] / topk_weights [K]
 * are optional (NULL to skip).  Replaces fused_moe_forward
 * (src/fused_moe.cu:233-263, declared src/fused_moe.cuh:28-32) and the
 * binding fused_moe_forward_torch (src/bindings.cpp:62-97). */
WR_API wr_status_t wr_fused_moe(const wr_moe_desc_t* desc, const void* x,
                         const void* gate_w, const void* weight_buf,
                         int64_t weight_buf_bytes, float* out,
                         int32_t* topk_ids, float* topk_weights,
                         void* workspace, size_t workspace_bytes,
                         wr_stream_t stream);

/* One decode token, exactly as wr_fused_moe, but with no workspace argument:
 * for callers that cannot allocate device memory (a host that owns the whole
 * device heap and gives the code it loads no workspace).  The scratch comes
 * from a 1 MiB array built into the library, which every GPU that loads the
 * library holds until the process exits; a layer that needs more (about
 * top_k * intermediate_dim * 4 + 8704 bytes) gets WR_ERR_UNSUPPORTED and
 * nothing is launched.  All calls on one device share the array and its
 * counters are cleared on `stream` before each launch, so calls that
 * overlap on the GPU race: serialise them.  The first call on each device
 * looks up the array's device address; make that call before any stream
 * capture.  A bounded wait that gives up inside a call sets the array's
 * status word, which the calls themselves never clear: read it with
 * wr_fused_moe_noalloc_status.  No counterpart in warp-route. */
WR_API wr_status_t wr_fused_moe_noalloc(const wr_moe_desc_t* desc, const void* x,
                                        const void* gate_w, const void* weight_buf,
                                        int64_t weight_buf_bytes, float* out,
                                        int32_t* topk_ids, float* topk_weights,
                                        wr_stream_t stream);
/* Reads (and clears) the status word of the built-in scratch that
 * wr_fused_moe_noalloc uses on the current device: WR_OK, or WR_ERR_TIMEOUT
 * when a bounded wait inside one of the calls since the last read gave up.
 * Synchronises `stream`; allocates nothing.  No counterpart in warp-route. */
WR_API wr_status_t wr_fused_moe_noalloc_status(wr_stream_t stream);

/* ---- fused layer, a batch of tokens ----------------------------------- */

/* num_tokens decode tokens: x [T,H] -> out [T,H] (fp32); topk_ids [T,K] and
 * topk_weights [T,K] optional.  Replaces batched_fused_moe_forward
 * (src/fused_moe_batched.cu:186-214, declared src/fused_moe_batched.cuh:29-33)
 * and batched_fused_moe_forward_torch (src/bindings.cpp:101-143). */
WR_API wr_status_t wr_batched_fused_moe(const wr_moe_desc_t* desc, int32_t num_tokens,
                                 const void* x, const void* gate_w,
                                 const void* weight_buf, int64_t weight_buf_bytes,
                                 float* out, int32_t* topk_ids,
                                 float* topk_weights, void* workspace,
                                 size_t workspace_bytes, wr_stream_t stream);

/* ---- tensor- / expert-parallel layer with a fused all-reduce ---------- */

/* Communicator of one rank for the all-reduce fused into the layer's last
 * step (no warp-route counterpart: warp-route is single-GPU; it replaces the
 * NCCL all-reduce a tensor- or expert-parallel caller would run after
 * fused_moe_forward).  Ranks are the GPUs of one node, one process each.
 * Set-up, once per process (allocates 8192 * hidden_dim + 256 bytes of
 * device memory on the current device):
 *   wr_comm_create -> wr_comm_get_handle -> exchange the world_size handles
 *   among the ranks (any host-side channel) -> wr_comm_open with all of them
 *   in rank order.
 * Every rank must then make the same sequence of wr_fused_moe_allreduce
 * calls.  A rank that stops makes the others' bounded waits for its partial
 * outputs give up after the peer timeout (2 s unless set with
 * wr_comm_set_peer_timeout_ns) instead of hanging: the call's output is then
 * wrong and wr_workspace_status reports WR_ERR_TIMEOUT.  After that the
 * ranks' launch counters differ and every later call would time out too:
 * recover with wr_comm_reset on every rank, between two host barriers, with
 * no layer call in flight (or destroy and recreate the communicators). */
typedef struct wr_comm* wr_comm_t;

/* Bytes of one rank's handle (a CUDA IPC memory handle). */
WR_API size_t wr_comm_handle_bytes(void);
WR_API wr_status_t wr_comm_create(int32_t rank, int32_t world_size, int32_t hidden_dim,
                                  wr_comm_t* out);
WR_API wr_status_t wr_comm_get_handle(wr_comm_t comm, void* handle);
/* handles: world_size * wr_comm_handle_bytes() bytes, rank order. */
WR_API wr_status_t wr_comm_open(wr_comm_t comm, const void* handles);
WR_API wr_status_t wr_comm_destroy(wr_comm_t comm);
/* Bound of each wait for a peer rank's partial outputs, in ns (0: the
 * default, 2 s).  Takes effect from the next call; a CUDA graph keeps the
 * bound its launches were captured with. */
WR_API wr_status_t wr_comm_set_peer_timeout_ns(wr_comm_t comm, uint64_t ns);
/* Puts this rank's launch counter and mailbox back to their initial state
 * (zero), on `stream`, and synchronises it.  After a call that timed out on
 * any rank: every rank waits at a host barrier until no layer call of any
 * rank is in flight, calls wr_comm_reset, and waits at a second host barrier
 * before its next wr_fused_moe_allreduce (no rank may store into a mailbox
 * that its owner has not reset yet).  The current device must be the
 * communicator's. */
WR_API wr_status_t wr_comm_reset(wr_comm_t comm, wr_stream_t stream);

/* num_tokens tokens through this rank's shard of the layer (a tensor-
 * parallel slice of every expert's intermediate dimension, or an
 * expert-parallel set of experts via desc->ep_*), with the ranks' partial
 * outputs summed in rank order inside the same kernel: out [T,H] fp32 holds
 * the full layer output, bit-identical on every rank.  Same arguments as
 * wr_batched_fused_moe plus the communicator (desc->hidden_dim must equal
 * the communicator's).  No warp-route counterpart (see wr_comm_t). */
WR_API wr_status_t wr_fused_moe_allreduce(const wr_moe_desc_t* desc, int32_t num_tokens,
                                          const void* x, const void* gate_w,
                                          const void* weight_buf, int64_t weight_buf_bytes,
                                          float* out, int32_t* topk_ids, float* topk_weights,
                                          void* workspace, size_t workspace_bytes,
                                          wr_comm_t comm, wr_stream_t stream);

/* ---- one layer of a decode stack --------------------------------------- */

/* The layer with the residual connection of a decode stack fused into its
 * last step: out = x + layer(x) in fp32 (with comm: the sum over the ranks'
 * shards first, exactly as wr_fused_moe_allreduce), and, when next_x is not
 * NULL, next_x = out rounded to desc->dtype (round to nearest even): the
 * next layer's input, written by the same kernel.  This is the arithmetic of
 * `h = (h.float() + layer(h)).to(dtype)`, bit for bit, without the two extra
 * kernels a plain decode loop launches per layer.  x [T,H] and next_x [T,H]
 * in desc->dtype (next_x must not alias x), out [T,H] fp32, the other
 * arguments as wr_batched_fused_moe; comm may be NULL (one GPU).  Shapes
 * that only the multi-kernel path takes (misaligned pointers, H or I not a
 * multiple of 16 bytes of elements) get WR_ERR_UNSUPPORTED.  No warp-route
 * counterpart: warp-route runs one layer per call and leaves the residual to
 * the caller (the per-layer launch overhead its README.md:17 cites). */
WR_API wr_status_t wr_moe_decode_layer(const wr_moe_desc_t* desc, int32_t num_tokens,
                                       const void* x, const void* gate_w,
                                       const void* weight_buf, int64_t weight_buf_bytes,
                                       float* out, void* next_x, int32_t* topk_ids,
                                       float* topk_weights, void* workspace,
                                       size_t workspace_bytes, wr_comm_t comm,
                                       wr_stream_t stream);

/* ---- weight packing ---------------------------------------------------- */

/* Packs one rank's shard of the expert weights into the flat layout (see
 * wr_expert_offsets) on the device, in one launch on `stream`: experts
 * [ep_first, ep_first + ep_num) of num_experts, renumbered from slot 0, and
 * of each the intermediate rows [tp_rank * I/tp_size, (tp_rank+1) * I/tp_size)
 * of gate and up and the matching columns of down, packed with
 * intermediate_dim = I / tp_size.  gate, up, down: host arrays of num_experts
 * device pointers to row-major [I,H], [I,H], [H,I] matrices of `dtype`
 * (entries outside the shard may be NULL).  dst: ep_num * expert stride
 * bytes (dst_bytes); the stride-rounding bytes are zeroed.  ep_num <= 64.
 * Replaces _pack_expert_weights (warp_route/functional.py:21-57), which
 * packs the whole layer with one copy per matrix and has no per-rank
 * slicing; the whole layer is ep_first = 0, ep_num = num_experts,
 * tp_rank = 0, tp_size = 1. */
WR_API wr_status_t wr_pack_experts(int32_t num_experts, int32_t hidden_dim,
                                   int32_t intermediate_dim, int32_t dtype, int32_t ep_first,
                                   int32_t ep_num, int32_t tp_rank, int32_t tp_size,
                                   const void* const* gate, const void* const* up,
                                   const void* const* down, void* dst, int64_t dst_bytes,
                                   wr_stream_t stream);

/* ---- naive multi-kernel layer ----------------------------------------- */

/* Scratch bytes for wr_naive_moe.  Replaces naive_moe_alloc_scratch /
 * NaiveMoEScratch (src/naive_moe.cu:24-33, src/naive_moe.cuh:25-32); the
 * caller allocates, so the call itself allocates nothing. */
WR_API size_t wr_naive_moe_workspace_size(const wr_moe_desc_t* desc);

/* Unfused layer, one kernel per step (router, top-K, gate, up, SwiGLU, down,
 * weighted accumulate).  Top-K runs on the device, so unlike warp-route there
 * is no mid-forward host synchronisation.  Replaces naive_moe_forward
 * (src/naive_moe.cu:181-241, declared src/naive_moe.cuh:39-44) and
 * naive_moe_forward_torch (src/bindings.cpp:26-59). */
WR_API wr_status_t wr_naive_moe(const wr_moe_desc_t* desc, const void* x,
                         const void* gate_w, const void* weight_buf,
                         int64_t weight_buf_bytes, float* out,
                         void* workspace, size_t workspace_bytes,
                         wr_stream_t stream);

/* ---- device status ----------------------------------------------------- */

/* Reads (and clears) the status word a fused call left in its workspace:
 * WR_OK, or WR_ERR_TIMEOUT when a bounded wait inside a kernel gave up.
 * Synchronises `stream`.  No warp-route counterpart (warp-route kernels have
 * no bounded waits). */
WR_API wr_status_t wr_workspace_status(void* workspace, wr_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* WARP_ROUTE_B200_H */
