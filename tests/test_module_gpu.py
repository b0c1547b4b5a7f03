"""GPU: warp_route.MoELayer, the module users call (warp_route/__init__.py:
10-105 of warp-route; its own test drives it the same way,
tests/test_python.py:51-106), against the CPU oracle.

Bar: expert indices bit-exact (checked through the router entry point on the
module's own weights), output within relative L2 1e-3 of the oracle.  Also:
writes into the parameters — in place, through `.data` (the usual
checkpoint-loading idiom), by load_state_dict — change the next forward's
output, because the parameters are the packed buffer the kernel reads.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import warp_route
from wr_testlib import host_array

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _oracle_out(layer, x):
    E, H, I, K = layer.num_experts, layer.hidden_dim, layer.intermediate_dim, layer.top_k
    buf = layer._pack_weights()
    xa = host_array(x.to(buf.dtype)).reshape(-1, H)
    gwa = host_array(layer.router.data)
    o_out, o_ids, _ = oracle.moe(xa, gwa, buf.view(torch.uint8).cpu().numpy(), E, H, I, K)
    return o_out, o_ids


def _check(layer, x, out):
    o_out, o_ids = _oracle_out(layer, x)
    err = oracle.rel_l2(out.detach().cpu().numpy().reshape(o_out.shape), o_out)
    assert err <= REL_L2_TOL, f"rel L2 {err:.3e}"
    E, H, K = layer.num_experts, layer.hidden_dim, layer.top_k
    _, ids, _ = warp_route.router_topk(x.to(layer.router.dtype).reshape(-1, H).contiguous(),
                                       layer.router.data, E, H, K)
    np.testing.assert_array_equal(ids.cpu().numpy(), o_ids)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("tokens", [0, 6])  # 0: a 1-D [H] token
def test_moelayer_forward_matches_oracle(dtype, tokens):
    torch.manual_seed(3)
    E, H, I, K = 8, 512, 1024, 4
    layer = warp_route.MoELayer(E, H, I, top_k=K, dtype=dtype).cuda()
    # larger weights than the 0.02 init so the outputs are well above rounding noise
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0.0, 0.05)
    x = torch.randn(H, device="cuda") if tokens == 0 else torch.randn(tokens, H, device="cuda")
    out = layer(x)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and out.shape == x.shape
    _check(layer, x, out)


def test_moelayer_sees_writes_through_data_and_state_dict():
    torch.manual_seed(4)
    E, H, I, K = 8, 512, 1024, 2
    layer = warp_route.MoELayer(E, H, I, top_k=K, dtype=torch.bfloat16).cuda()
    x = torch.randn(H, device="cuda")
    before = layer(x).clone()
    _, ids, _ = warp_route.router_topk(x.to(torch.bfloat16), layer.router.data, E, H, K)
    e = int(ids.view(-1)[0])  # an expert this token uses
    buf = layer._pack_weights()
    # the checkpoint-loading idiom: a write through .data
    w = torch.randn(I, H, device="cuda", dtype=torch.bfloat16) * 0.05
    layer.gate_proj[e].data.copy_(w)
    assert layer._pack_weights() is buf  # no repack: the parameter is the buffer
    after = layer(x)
    torch.cuda.synchronize()
    assert not torch.equal(after, before), "a write through .data did not reach the kernel"
    _check(layer, x, after)
    # load_state_dict writes in place too
    sd = {k: v.clone() for k, v in layer.state_dict().items()}
    sd[f"down_proj.{e}"] = torch.randn(H, I, device="cuda", dtype=torch.bfloat16) * 0.05
    layer.load_state_dict(sd)
    again = layer(x)
    torch.cuda.synchronize()
    assert not torch.equal(again, after)
    _check(layer, x, again)
