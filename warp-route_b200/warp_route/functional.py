"""Functional API of warp-route, backed by the B200-native kernels.

Drop-in for warp-route's warp_route/functional.py: the same names, positional
signatures and error behaviour (`_pack_expert_weights`, `fused_moe`,
`naive_moe`, `batched_fused_moe`), plus `fused_moe_batched` (alias of
`batched_fused_moe`) and a few keyword-only extras.

Differences a caller may notice (all additive):
  * float32 or bfloat16 inputs (x, gate_w and weight_buf share one dtype);
    the output is always float32 — bf16 rounding of the output alone would
    cost ~2e-3 relative error;
  * top_k may be anything in [1, num_experts] (num_experts <= 64);
  * calls are asynchronous on the current CUDA stream (warp-route calls
    cudaDeviceSynchronize after each launch);
  * optional `router_bias` (fp32 [E], added to the logits).
There is no CPU fallback: without the compiled extension every call raises.
"""
from __future__ import annotations

import functools
from typing import List, Optional, Tuple

import torch


@functools.lru_cache(maxsize=1)
def _load_extension():
    """Import warp_route._C (warp_route/functional.py:9-18 of warp-route)."""
    try:
        from . import _C  # noqa: F401  (built in-tree by warp-route_b200/build.py)
        return _C
    except ImportError as e:
        raise ImportError(
            "warp_route._C extension not found or failed to load "
            f"({e}). Build it with: python warp-route_b200/build.py "
            "(requires nvcc for sm_100a and PyTorch)"
        ) from e


def _expert_stride_elems(hidden_dim: int, intermediate_dim: int, elt: int) -> int:
    raw = (2 * intermediate_dim * hidden_dim + hidden_dim * intermediate_dim) * elt
    return ((raw + 127) & ~127) // elt


def _pack_expert_weights(
    gate_proj: List[torch.Tensor],
    up_proj: List[torch.Tensor],
    down_proj: List[torch.Tensor],
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
) -> torch.Tensor:
    """Pack per-expert weights into the flat layout the kernels read.

    Per expert, row-major: [gate I x H][up I x H][down H x I]; each expert
    block starts on a 128-byte boundary (warp_route/functional.py:21-57 and
    src/expert_layout.cuh:34-47 of warp-route).  The buffer keeps the dtype of
    the inputs (float32 or bfloat16) and lives on gate_proj[0]'s device.
    """
    dtype = gate_proj[0].dtype
    if dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"expert weights must be float32 or bfloat16, got {dtype}")
    if _device_packable(gate_proj, up_proj, down_proj, num_experts):
        # one device launch for the whole buffer (wr_pack_experts)
        return _load_extension().pack_experts(list(gate_proj), list(up_proj), list(down_proj),
                                               num_experts, hidden_dim, intermediate_dim, 0,
                                               num_experts, 0, 1)
    elt = torch.empty((), dtype=dtype).element_size()
    n = intermediate_dim * hidden_dim
    stride = _expert_stride_elems(hidden_dim, intermediate_dim, elt)
    device = gate_proj[0].device
    buf = torch.zeros(num_experts * stride, dtype=dtype, device=device)
    for e in range(num_experts):
        base = e * stride
        buf[base:base + n] = gate_proj[e].contiguous().view(-1).to(dtype)
        buf[base + n:base + 2 * n] = up_proj[e].contiguous().view(-1).to(dtype)
        buf[base + 2 * n:base + 3 * n] = down_proj[e].contiguous().view(-1).to(dtype)
    return buf


def _device_packable(gate_proj, up_proj, down_proj, num_experts: int) -> bool:
    """All matrices CUDA, contiguous, of one dtype and device, and at most 64
    experts: the device pack kernel takes them as they are."""
    if num_experts > 64:
        return False
    ref = gate_proj[0]
    if not ref.is_cuda:
        return False
    for lst in (gate_proj, up_proj, down_proj):
        if len(lst) != num_experts:
            return False
        for t in lst:
            if not (t.is_cuda and t.is_contiguous() and t.dtype == ref.dtype
                    and t.device == ref.device and t.dim() == 2):
                return False
    return True


def pack_expert_shard(
    gate_proj: List[torch.Tensor],
    up_proj: List[torch.Tensor],
    down_proj: List[torch.Tensor],
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    *,
    tp_rank: int = 0,
    tp_size: int = 1,
    ep_rank: int = 0,
    ep_size: int = 1,
) -> Tuple[torch.Tensor, int, int, int]:
    """One rank's shard of the layer, packed on the device in one launch.

    Expert parallel: rank ep_rank of ep_size holds experts
    [ep_rank*E/ep_size, (ep_rank+1)*E/ep_size), packed from slot 0.  Tensor
    parallel: rank tp_rank of tp_size holds, of every expert, the intermediate
    rows [tp_rank*I/tp_size, (tp_rank+1)*I/tp_size) of gate and up and the
    matching columns of down.  The per-expert matrices (CUDA, contiguous,
    float32 or bfloat16: gate/up [I,H], down [H,I]) stay where they are; only
    the shard's experts are read.  Returns (weight_buf, ep_first_expert,
    ep_num_local, intermediate_local): pass the last three to the fused entry
    points (ep_num_local = 0 when the rank holds every expert).
    """
    if ep_size < 1 or num_experts % ep_size or not 0 <= ep_rank < ep_size:
        raise ValueError(f"ep_size {ep_size} must divide num_experts {num_experts} "
                         f"and 0 <= ep_rank < ep_size")
    if tp_size < 1 or intermediate_dim % tp_size or not 0 <= tp_rank < tp_size:
        raise ValueError(f"tp_size {tp_size} must divide intermediate_dim {intermediate_dim} "
                         f"and 0 <= tp_rank < tp_size")
    n = num_experts // ep_size
    first = ep_rank * n
    buf = _load_extension().pack_experts(list(gate_proj), list(up_proj), list(down_proj),
                                         num_experts, hidden_dim, intermediate_dim, first, n,
                                         tp_rank, tp_size)
    return buf, (first if ep_size > 1 else 0), (n if ep_size > 1 else 0), intermediate_dim // tp_size


def fused_moe(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    weight_buf: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    top_k: int,
    *,
    router_bias: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One decode token: x [hidden_dim] -> float32 [hidden_dim]."""
    _C = _load_extension()
    if router_bias is None:
        return _C.fused_moe_forward(x, gate_w, weight_buf, num_experts, hidden_dim,
                                    intermediate_dim, top_k)
    if x.dim() != 1:
        raise ValueError(f"fused_moe expects 1D input [hidden], got shape {tuple(x.shape)}")
    return _C.fused_moe_routed(x, gate_w, weight_buf, num_experts, hidden_dim,
                               intermediate_dim, top_k, router_bias)[0]


def naive_moe(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    weight_buf: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    top_k: int,
) -> torch.Tensor:
    """One decode token through the unfused kernel-per-step path."""
    _C = _load_extension()
    return _C.naive_moe_forward(x, gate_w, weight_buf, num_experts, hidden_dim,
                                intermediate_dim, top_k)


def batched_fused_moe(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    weight_buf: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    top_k: int,
    *,
    router_bias: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Decode batch: x [batch, hidden_dim] -> float32 [batch, hidden_dim]."""
    if x.dim() != 2:
        raise ValueError(f"batched_fused_moe expects 2D input [batch, hidden], got shape {x.shape}")
    batch_size, hd = x.shape
    if hd != hidden_dim:
        raise ValueError(f"Input hidden dim {hd} does not match hidden_dim={hidden_dim}")
    _C = _load_extension()
    if router_bias is None:
        return _C.batched_fused_moe_forward(x, gate_w, weight_buf, num_experts, hidden_dim,
                                            intermediate_dim, top_k)
    return _C.fused_moe_routed(x, gate_w, weight_buf, num_experts, hidden_dim,
                               intermediate_dim, top_k, router_bias)[0]


# The name used by the batched benchmark configuration.
fused_moe_batched = batched_fused_moe


def fused_moe_routed(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    weight_buf: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    top_k: int,
    *,
    router_bias: Optional[torch.Tensor] = None,
    ep_first_expert: int = 0,
    ep_num_local: int = 0,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Layer output plus its routing: (out fp32, expert ids int32 [T,K],
    weights fp32 [T,K]).  x is [H] or [T,H].  With ep_num_local > 0 the
    weight_buf holds experts [ep_first_expert, ep_first_expert + ep_num_local)
    only, and the output is this shard's partial sum."""
    _C = _load_extension()
    return _C.fused_moe_routed(x, gate_w, weight_buf, num_experts, hidden_dim,
                               intermediate_dim, top_k, router_bias, ep_first_expert,
                               ep_num_local)


def router_topk(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    top_k: int,
    *,
    router_bias: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Router only: (logits fp32 [T,E], ids int32 [T,K], weights fp32 [T,K])."""
    _C = _load_extension()
    return _C.router_topk(x, gate_w, num_experts, hidden_dim, top_k, router_bias)


def exchange_handles(mine: bytes, group=None) -> bytes:
    """Every rank's handle bytes, concatenated in rank order (collective over
    `group`; every handle must have the same length)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    handles: List[Optional[bytes]] = [None] * world
    dist.all_gather_object(handles, mine, group=group)
    if any(h is None or len(h) != len(mine) for h in handles):
        raise RuntimeError("communicator handles of different sizes")
    return b"".join(handles)


class PeerComm:
    """One rank's communicator for the all-reduce fused into the layer.

    Tensor- or expert-parallel layers on the GPUs of one node, one process
    per GPU: each rank streams its shard of the weights and the ranks'
    partial outputs are summed (rank order, identical on every rank) in the
    same kernel, over NVLink peer memory, instead of a separate NCCL
    all-reduce.  Construction is collective over `group` (the ranks exchange
    CUDA IPC handles through torch.distributed); every rank must then make
    the same sequence of `fused_moe_allreduce` calls.  No warp-route
    counterpart (warp-route is single-GPU).
    """

    def __init__(self, hidden_dim: int, group=None):
        import torch.distributed as dist

        _C = _load_extension()
        self.rank = dist.get_rank(group)
        self.world_size = dist.get_world_size(group)
        self.hidden_dim = hidden_dim
        self._ptr = _C.comm_create(self.rank, self.world_size, hidden_dim)
        all_handles = exchange_handles(bytes(_C.comm_handle(self._ptr).numpy()), group)
        _C.comm_open(self._ptr, torch.frombuffer(bytearray(all_handles), dtype=torch.uint8))

    @property
    def handle(self) -> int:
        if self._ptr == 0:
            raise RuntimeError("communicator is closed")
        return self._ptr

    def set_peer_timeout(self, seconds: float) -> None:
        """Bound of each wait for another rank's partial outputs (default
        2 s; 0 restores it).  A call whose wait gives up returns a wrong
        output and leaves WR_ERR_TIMEOUT in its workspace status."""
        _load_extension().comm_set_peer_timeout_ns(self.handle, int(seconds * 1e9))

    def reset(self, group=None) -> None:
        """Recovery after a call timed out on any rank (collective over
        `group`): once no rank has a layer call in flight, every rank puts its
        launch counter and mailbox back to zero, between two barriers, so the
        ranks' launches are numbered alike again."""
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(group)
        _load_extension().comm_reset(self.handle)
        dist.barrier(group)

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (call on every
        rank, after the last layer call has finished)."""
        if self._ptr:
            _load_extension().comm_destroy(self._ptr)
            self._ptr = 0


def moe_decode_layer(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    weight_buf: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    top_k: int,
    *,
    next_x: Optional[torch.Tensor] = None,
    comm: Optional["PeerComm"] = None,
    router_bias: Optional[torch.Tensor] = None,
    ep_first_expert: int = 0,
    ep_num_local: int = 0,
) -> torch.Tensor:
    """One layer of a decode stack with the residual connection fused into
    the layer kernel's last step: returns out = x + layer(x) (float32; with
    `comm`, the layer is this rank's shard and the sum over the ranks comes
    first) and, if `next_x` is given (x's shape and dtype, not x itself),
    writes next_x = out.to(x.dtype) — the next layer's input — from the same
    kernel.  Bit-identical to `(x.float() + layer(x)).to(x.dtype)`, with no
    extra kernels per layer."""
    _C = _load_extension()
    return _C.moe_decode_layer(x, gate_w, weight_buf, num_experts, hidden_dim,
                               intermediate_dim, top_k, comm.handle if comm is not None else 0,
                               router_bias, ep_first_expert, ep_num_local, next_x)


def fused_moe_allreduce(
    x: torch.Tensor,
    gate_w: torch.Tensor,
    weight_buf: torch.Tensor,
    num_experts: int,
    hidden_dim: int,
    intermediate_dim: int,
    top_k: int,
    comm: PeerComm,
    *,
    router_bias: Optional[torch.Tensor] = None,
    ep_first_expert: int = 0,
    ep_num_local: int = 0,
    return_routing: bool = False,
):
    """This rank's shard of the layer with every rank's output summed in the
    same kernel: x [H] or [T,H] -> float32, the full layer output on every
    rank.  weight_buf holds this rank's shard: a tensor-parallel slice
    (intermediate_dim = this rank's columns) or, with ep_num_local > 0, the
    experts [ep_first_expert, ep_first_expert + ep_num_local).  With
    return_routing=True the result is (out, expert ids int32 [T,K], weights
    fp32 [T,K]), the routing being identical on every rank."""
    _C = _load_extension()
    res = _C.fused_moe_allreduce(x, gate_w, weight_buf, num_experts, hidden_dim,
                                 intermediate_dim, top_k, comm.handle, router_bias,
                                 ep_first_expert, ep_num_local)
    return res if return_routing else res[0]
