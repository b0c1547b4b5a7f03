"""CPU: pin the oracle against warp-route's own composition.

The fixture holds outputs, indices and weights of `torch_moe_reference`
(tests/test_python.py:15-37 of warp-route) on the reference's own test
configurations (tests/test_python.py:116-125, tests/test_batched.py:75-79),
the benchmark's tiny CPU configuration, and bf16-rounded variants.
"""
from __future__ import annotations

import numpy as np
import pytest

import inputs as gi
import oracle
from conftest import golden_inputs, golden_selected, load_golden

_, INDEX = load_golden()


@pytest.mark.parametrize("meta", INDEX, ids=[m["name"] for m in INDEX])
def test_oracle_matches_reference(golden, meta):
    z, _ = golden
    x, gw, ex = golden_inputs(meta)
    if meta["bf16"]:
        xa, gwa = gi.bf16_bits(x), gi.bf16_bits(gw)
    else:
        xa, gwa = x.numpy().astype(np.float32), gw.numpy().astype(np.float32)
    # only the experts the reference selected are read (the rest stay zero, so
    # a wrong selection would also show as a wrong output)
    wb = gi.pack_numpy(ex, bf16=meta["bf16"], only=golden_selected(z, meta))
    out, ids, w = oracle.moe(np.ascontiguousarray(xa), np.ascontiguousarray(gwa), wb, meta["E"],
                             meta["H"], meta["I"], meta["top_k"])
    name = meta["name"]
    np.testing.assert_array_equal(ids, z[name + "/ids"])
    np.testing.assert_allclose(w, z[name + "/weights"], rtol=1e-5, atol=1e-7)
    # fp64-accumulated oracle vs the reference's fp32 torch matmuls.
    assert oracle.rel_l2(out, z[name + "/out"]) < 1e-5


def test_oracle_router_matches_torch_selection(golden):
    """The logit-order selection agrees with the reference's probs-order
    torch.topk on every golden token."""
    z, index = golden
    for meta in index:
        x, gw, _ = golden_inputs(meta, experts=False)
        if meta["bf16"]:
            xa, gwa = gi.bf16_bits(x), gi.bf16_bits(gw)
        else:
            xa, gwa = x.numpy(), gw.numpy()
        _, ids, _ = oracle.router(np.ascontiguousarray(xa), np.ascontiguousarray(gwa),
                                  meta["top_k"])
        np.testing.assert_array_equal(ids, z[meta["name"] + "/ids"])
