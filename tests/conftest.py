"""Shared pytest setup: paths, the `gpu` marker, golden fixtures."""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("warp-route_b200", "oracle", os.path.join("tests", "golden")):
    p = os.path.join(REPO, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN_PATH = os.path.join(REPO, "tests", "golden", "reference_golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden():
    z = np.load(GOLDEN_PATH)
    index = json.loads(bytes(z["index_json"]).decode())
    return z, index


@pytest.fixture(scope="session")
def golden():
    return load_golden()


def golden_inputs(meta, experts=True):
    """Regenerate a golden case's CPU inputs and check them against the
    fixture's checksums.  Returns (x [T,H] torch fp32, gate_w, experts); for a
    bf16 case x and gate_w come rounded to bf16, while the experts stay fp32
    (gi.pack_numpy(..., bf16=True) rounds them).  experts=False skips them."""
    import inputs as gi

    E, H, I, T, seed = meta["E"], meta["H"], meta["I"], meta["tokens"], meta["seed"]
    if meta["gen"] == "reference_test_inputs":
        x, gw, ex = gi.reference_test_inputs(E, H, I, seed, experts=experts)
    elif meta["gen"] == "reference_batched_inputs":
        x, gw, ex = gi.reference_batched_inputs(E, H, I, T, seed, experts=experts)
    else:
        x, gw, ex = gi.baseline_inputs(E, H, I, seed, experts=experts)
    if meta["bf16"]:
        x, gw = gi.round_bf16(x), gi.round_bf16(gw)
    assert abs(gi.checksum(x) - meta["checksum_x"]) < 1e-6, "input generator drifted (x)"
    assert abs(gi.checksum(gw) - meta["checksum_gate_w"]) < 1e-6, "input generator drifted (gate_w)"
    return x.reshape(-1, H), gw, ex


def golden_selected(z, meta):
    """The experts the reference selected for any token of a golden case."""
    return set(int(e) for e in z[meta["name"] + "/ids"].reshape(-1))
