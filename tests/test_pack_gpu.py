"""GPU tests of the device-side weight packing (wr_pack_experts through
warp_route.pack_expert_shard and _pack_expert_weights): bit-identical to the
layout packed with plain torch copies (warp-route's _pack_expert_weights,
warp_route/functional.py:21-57), for the whole layer and for tensor- and
expert-parallel shards, and usable by the layer entry points."""
from __future__ import annotations

import pytest
import torch

import warp_route
from warp_route import functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _experts(E, H, I, dtype, seed=0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    mk = lambda r, c: (torch.randn(r, c, generator=g, device="cuda") / c ** 0.5).to(dtype)  # noqa: E731
    return ([mk(I, H) for _ in range(E)], [mk(I, H) for _ in range(E)],
            [mk(H, I) for _ in range(E)])


def _torch_pack(gate, up, down, experts, H, I, i0, Il, dtype):
    """The layout with plain torch copies: for each listed expert
    [gate rows i0..][up rows i0..][down cols i0..], stride rounded to 128 B."""
    elt = torch.empty((), dtype=dtype).element_size()
    stride = F._expert_stride_elems(H, Il, elt)
    buf = torch.zeros(len(experts) * stride, dtype=dtype, device="cuda")
    n = Il * H
    for j, e in enumerate(experts):
        b = j * stride
        buf[b:b + n] = gate[e][i0:i0 + Il].reshape(-1)
        buf[b + n:b + 2 * n] = up[e][i0:i0 + Il].reshape(-1)
        buf[b + 2 * n:b + 3 * n] = down[e][:, i0:i0 + Il].contiguous().reshape(-1)
    return buf


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("E,H,I", [(8, 256, 512), (3, 100, 52), (6, 200, 36)])
def test_whole_layer_matches_torch_copies(dtype, E, H, I):
    gate, up, down = _experts(E, H, I, dtype)
    got = warp_route._pack_expert_weights(gate, up, down, E, H, I)
    ref = _torch_pack(gate, up, down, list(range(E)), H, I, 0, I, dtype)
    torch.cuda.synchronize()
    assert got.dtype == dtype and torch.equal(got.view(torch.uint8), ref.view(torch.uint8))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("tp", [2, 4])
def test_tensor_parallel_shards(dtype, tp):
    E, H, I = 8, 256, 512
    gate, up, down = _experts(E, H, I, dtype, seed=1)
    for r in range(tp):
        buf, first, num, Il = F.pack_expert_shard(gate, up, down, E, H, I, tp_rank=r, tp_size=tp)
        assert (first, num, Il) == (0, 0, I // tp)
        ref = _torch_pack(gate, up, down, list(range(E)), H, I, r * Il, Il, dtype)
        torch.cuda.synchronize()
        assert torch.equal(buf.view(torch.uint8), ref.view(torch.uint8))


@pytest.mark.parametrize("ep", [2, 8])
def test_expert_parallel_shards(ep):
    E, H, I = 8, 256, 512
    gate, up, down = _experts(E, H, I, torch.bfloat16, seed=2)
    for r in range(ep):
        buf, first, num, Il = F.pack_expert_shard(gate, up, down, E, H, I, ep_rank=r, ep_size=ep)
        n = E // ep
        assert (first, num, Il) == (r * n, n, I)
        ref = _torch_pack(gate, up, down, list(range(r * n, (r + 1) * n)), H, I, 0, I,
                          torch.bfloat16)
        torch.cuda.synchronize()
        assert torch.equal(buf.view(torch.uint8), ref.view(torch.uint8))


def test_shards_run_the_layer():
    """TP x EP shards (2 x 2) packed on the device sum to the whole layer."""
    E, H, I, K, T = 8, 512, 1024, 2, 20
    gate, up, down = _experts(E, H, I, torch.bfloat16, seed=3)
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    gw = (torch.randn(E, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    whole = warp_route._pack_expert_weights(gate, up, down, E, H, I)
    ref = F.batched_fused_moe(x, gw, whole, E, H, I, K)
    acc = torch.zeros_like(ref)
    for tr in range(2):
        for er in range(2):
            buf, first, num, Il = F.pack_expert_shard(gate, up, down, E, H, I, tp_rank=tr,
                                                      tp_size=2, ep_rank=er, ep_size=2)
            out, _, _ = F.fused_moe_routed(x, gw, buf, E, H, Il, K, ep_first_expert=first,
                                           ep_num_local=num)
            acc += out
    torch.cuda.synchronize()
    err = (torch.linalg.vector_norm((acc - ref).double()) /
           torch.linalg.vector_norm(ref.double())).item()
    assert err <= 1e-5, err


def test_bad_shard_shapes_raise():
    E, H, I = 4, 128, 256
    gate, up, down = _experts(E, H, I, torch.float32, seed=4)
    with pytest.raises(ValueError):
        F.pack_expert_shard(gate, up, down, E, H, I, tp_size=3)
    with pytest.raises(ValueError):
        F.pack_expert_shard(gate, up, down, E, H, I, ep_size=3)
    bad = list(down)
    bad[1] = bad[1].t().contiguous()  # [I, H] instead of [H, I]
    with pytest.raises(RuntimeError, match="down_proj"):
        F.pack_expert_shard(gate, up, bad, E, H, I)
