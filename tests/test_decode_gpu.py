"""GPU tests of the decode-step driver (warp_route.decode.MoEStack) and of the
layer entry point it is built on (moe_decode_layer / wr_moe_decode_layer,
the residual connection fused into the layer kernel's last step).

  * the fused residual equals the unfused composition
    `(x.float() + layer(x)).to(dtype)` bit for bit — out and the next
    input — for one token (streaming kernel), a bf16 batch (grouped tcgen05
    path), fp32 token blocks and a one-rank communicator (the fused
    all-reduce tail);
  * the graph replay equals the same stack run eagerly bit for bit, every
    step, for a single token and a batch;
  * the chained stack follows the CPU oracle: each layer's MoE part within
    the suite's relative L2 1e-3 of the oracle on the GPU chain's own input,
    and the whole chain within 1e-3 of the oracle chain that rounds the
    residual to bf16 at the same points.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from warp_route import functional as F
from warp_route import synthetic
from warp_route.decode import MoEStack, StackLayer
from wr_testlib import host_array

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _stack(E, H, I, K, T, n_layers, seed=50, **kw):
    layers = []
    for li in range(n_layers):
        L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=seed + li, layer=li,
                                 router_bias=True)
        layers.append(StackLayer(L.gate_w, L.weight_buf, L.router_bias))
    return MoEStack(layers, E, H, I, K, T, **kw)


@pytest.mark.parametrize("T,dtype,one_rank", [(1, torch.bfloat16, False),
                                              (16, torch.bfloat16, False),
                                              (3, torch.float32, False),
                                              (1, torch.bfloat16, True),
                                              (16, torch.bfloat16, True)])
def test_fused_residual_equals_unfused(T, dtype, one_rank):
    E, H, I, K = 8, 512, 1024, 2
    L = synthetic.make_layer(E, H, I, K, dtype=dtype, seed=61, tokens=T, router_bias=True)
    x = L.x
    nxt = torch.empty_like(x)
    comm = None
    _C = F._load_extension()
    if one_rank:
        handle = _C.comm_create(0, 1, H)
        comm = type("OneRank", (), {"handle": handle})()
    try:
        for _ in range(2):
            out = F.moe_decode_layer(x, L.gate_w, L.weight_buf, E, H, I, K, next_x=nxt,
                                     comm=comm, router_bias=L.router_bias)
            layer = F.fused_moe_routed(x, L.gate_w, L.weight_buf, E, H, I, K,
                                       router_bias=L.router_bias)[0]
            ref = x.float() + layer
            torch.cuda.synchronize()
            assert torch.equal(out, ref), "fused residual differs from x.float() + layer(x)"
            assert torch.equal(nxt, ref.to(dtype)), "next input differs from the rounded sum"
    finally:
        if one_rank:
            _C.comm_destroy(handle)
    assert _C.workspace_status(x) == 0


def test_fused_residual_rejects_aliasing():
    E, H, I, K = 8, 512, 1024, 2
    L = synthetic.make_layer(E, H, I, K, dtype=torch.bfloat16, seed=62)
    with pytest.raises(RuntimeError, match="alias"):
        F.moe_decode_layer(L.x, L.gate_w, L.weight_buf, E, H, I, K, next_x=L.x)


@pytest.mark.parametrize("T", [1, 16])
def test_graph_replay_equals_eager(T):
    E, H, I, K = 8, 512, 1024, 2
    stack = _stack(E, H, I, K, T, 4)
    g = torch.Generator(device="cuda")
    g.manual_seed(T)
    shape = (H,) if T == 1 else (T, H)
    for step in range(3):
        x = torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)
        ref = stack.eager(x)
        got = stack.step(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"step {step}: graph replay differs from the eager stack"
        assert torch.isfinite(got.float()).all()
    stack.close()


def test_capture_waits_for_work_queued_on_the_callers_stream():
    """The first step() captures the graph after warm-up runs on its own
    stream; those runs write the stack's static buffers, so they must wait
    for an eager call still queued on the caller's stream (held back here by
    a sleep kernel ahead of it)."""
    E, H, I, K, T = 8, 512, 1024, 2, 1
    stack = _stack(E, H, I, K, T, 4, seed=90)
    x = torch.randn(H, device="cuda").to(torch.bfloat16)
    torch.cuda._sleep(50_000_000)  # ~25 ms of device time ahead of the eager stack
    ref = stack.eager(x)
    got = stack.step(x).clone()
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    stack.close()


def test_external_all_reduce_path_equals_fused():
    """A stack given an external collective (here the identity: one rank)
    adds the residual after it; the result equals the fused stack's."""
    E, H, I, K, T = 8, 512, 1024, 2, 1
    fused = _stack(E, H, I, K, T, 3, seed=80)
    ext = MoEStack(fused.layers, E, H, I, K, T, all_reduce=lambda t: None)
    x = torch.randn(H, device="cuda").to(torch.bfloat16)
    a = fused.eager(x)
    b = ext.eager(x)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("T", [1, 16])
def test_chain_follows_the_oracle(T):
    E, H, I, K = 8, 512, 1024, 2
    n_layers = 3
    stack = _stack(E, H, I, K, T, n_layers, seed=70)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    shape = (H,) if T == 1 else (T, H)
    x = torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)
    got = stack.step(x).clone()
    # layer by layer on the GPU chain's own inputs
    h = x.clone()
    nxt = torch.empty_like(h)
    for i, L in enumerate(stack.layers):
        out = stack.layer(i, h, nxt)
        torch.cuda.synchronize()
        wb = L.weight_buf.cpu().view(torch.uint8).numpy()
        o_out, _, _ = oracle.moe(host_array(h).reshape(-1, H), host_array(L.gate_w), wb, E, H, I,
                                 K, L.router_bias.cpu().numpy())
        moe_part = (out - h.float()).cpu().numpy().reshape(o_out.shape)
        err = oracle.rel_l2(moe_part, o_out)
        assert err <= REL_L2_TOL, f"layer {i}: rel L2 {err:.3e}"
        h, nxt = nxt.clone(), torch.empty_like(nxt)
    assert torch.equal(h, got), "the graph step differs from the layer-by-layer chain"
    # the whole chain against the oracle chain: h <- bf16(h + moe(h)) per layer
    hc = x.cpu()
    for L in stack.layers:
        wb = L.weight_buf.cpu().view(torch.uint8).numpy()
        o_out, _, _ = oracle.moe(host_array(hc).reshape(-1, H), host_array(L.gate_w), wb, E, H,
                                 I, K, L.router_bias.cpu().numpy())
        hc = (hc.float() + torch.from_numpy(np.asarray(o_out)).reshape(hc.shape)).to(
            torch.bfloat16)
    err = oracle.rel_l2(got.float().cpu().numpy(), hc.float().numpy())
    assert err <= REL_L2_TOL, f"chain rel L2 {err:.3e}"
    stack.close()
