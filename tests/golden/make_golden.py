"""Generate tests/golden/reference_golden.npz from warp-route's own oracle.

Runs the reference's pure-torch composition `torch_moe_reference`
(tests/test_python.py:15-37 of warp-route), imported from a warp-route
checkout, on the reference's own test configurations:
  - tests/test_python.py:116-125   (7 single-token configs, seed 42),
  - tests/test_batched.py:75-79    (batched configs, seed 42; the reference
                                    compares against a loop of single-token
                                    calls, so the golden is the composition
                                    applied per token),
  - the benchmark's tiny CPU configuration (H512 I1024 E8 k2, seed 0),
plus bf16-rounded variants (inputs rounded to bf16, composition run in fp32),
and cases the reference's CUDA kernels cannot run but its composition can:
  - top_k 4, 6 and 8 (the fused kernels stop at 2, src/bindings.cpp:75,117),
    on the single-token test inputs with E up to 64;
  - bf16-rounded token batches (the grouped tensor-core path of this build):
    E8 k2 B16, E16 k4 B64, E64 k6 B5;
  - the DeepSeek-shaped benchmark layer (H2048 I1408 E64 k6, the benchmark
    init with seed 0, bf16-rounded).

Indices and weights are taken with the same torch ops the composition uses
(gate_w @ x, softmax, torch.topk).  The reference checkout is needed only
here; the fixture it writes is committed and travels.

Usage:  python tests/golden/make_golden.py --reference <warp-route checkout>
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs as gi  # noqa: E402

SINGLE = [(8, 256, 512, 1), (8, 256, 512, 2), (8, 512, 1024, 1), (8, 512, 1024, 2),
          (16, 256, 512, 1), (16, 256, 512, 2), (8, 1024, 2048, 2)]
BATCHED = [(8, 256, 512, 1, b) for b in (1, 4, 16, 64)] + \
          [(8, 256, 512, 2, b) for b in (1, 4, 16, 64)] + \
          [(16, 512, 1024, 2, b) for b in (1, 4, 16)]
BF16_SINGLE = [(8, 512, 1024, 2), (16, 256, 512, 2), (8, 1024, 2048, 2)]
TOPK_SINGLE = [(8, 256, 512, 4), (16, 256, 512, 6), (16, 512, 1024, 8), (64, 256, 512, 6),
               (64, 512, 1024, 8)]
BF16_BATCHED = [(8, 512, 1024, 2, 16), (16, 512, 1024, 4, 64), (64, 256, 512, 6, 5)]
DEEPSEEK = (64, 2048, 1408, 6)


def load_reference(ref_root: str):
    sys.path.insert(0, ref_root)
    sys.path.insert(0, os.path.join(ref_root, "tests"))
    import test_python  # the reference's test module; its top-level import is torch-only
    return test_python.torch_moe_reference


def select(x: torch.Tensor, gate_w: torch.Tensor, k: int):
    probs = torch.softmax(gate_w @ x, dim=0)
    w, idx = torch.topk(probs, k)
    return idx.numpy().astype(np.int32), w.numpy().astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="warp-route checkout (read-only)")
    ap.add_argument("--out", default=os.path.join(HERE, "reference_golden.npz"))
    args = ap.parse_args()
    ref = load_reference(args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    arrays = {}
    index = []

    def emit(name, meta, x, gate_w, experts, k):
        xs = x.reshape(-1, x.shape[-1])
        outs, ids, ws = [], [], []
        for t in range(xs.shape[0]):
            outs.append(ref(xs[t].clone(), gate_w, *experts, k).numpy().astype(np.float32))
            i, w = select(xs[t], gate_w, k)
            ids.append(i)
            ws.append(w)
        arrays[name + "/out"] = np.stack(outs)
        arrays[name + "/ids"] = np.stack(ids)
        arrays[name + "/weights"] = np.stack(ws)
        meta = dict(meta, name=name, top_k=k,
                    checksum_x=gi.checksum(x), checksum_gate_w=gi.checksum(gate_w),
                    checksum_experts=gi.checksum(*experts[0], *experts[1], *experts[2]))
        index.append(meta)

    for (E, H, I, k) in SINGLE:
        x, gw, ex = gi.reference_test_inputs(E, H, I, 42)
        emit(f"single_E{E}_H{H}_I{I}_k{k}",
             dict(kind="single", gen="reference_test_inputs", E=E, H=H, I=I, seed=42,
                  tokens=1, bf16=False), x, gw, ex, k)
    for (E, H, I, k, B) in BATCHED:
        x, gw, ex = gi.reference_batched_inputs(E, H, I, B, 42)
        emit(f"batched_E{E}_H{H}_I{I}_k{k}_B{B}",
             dict(kind="batched", gen="reference_batched_inputs", E=E, H=H, I=I, seed=42,
                  tokens=B, bf16=False), x, gw, ex, k)
    x, gw, ex = gi.baseline_inputs(8, 512, 1024, 0)
    emit("tiny_E8_H512_I1024_k2",
         dict(kind="tiny", gen="baseline_inputs", E=8, H=512, I=1024, seed=0, tokens=1,
              bf16=False), x, gw, ex, 2)
    for (E, H, I, k) in BF16_SINGLE:
        x, gw, ex = gi.reference_test_inputs(E, H, I, 42)
        rb = gi.round_bf16
        x, gw = rb(x), rb(gw)
        ex = tuple([rb(t) for t in lst] for lst in ex)
        emit(f"bf16_E{E}_H{H}_I{I}_k{k}",
             dict(kind="single", gen="reference_test_inputs", E=E, H=H, I=I, seed=42,
                  tokens=1, bf16=True), x, gw, ex, k)

    for (E, H, I, k) in TOPK_SINGLE:
        x, gw, ex = gi.reference_test_inputs(E, H, I, 42)
        emit(f"topk_E{E}_H{H}_I{I}_k{k}",
             dict(kind="single", gen="reference_test_inputs", E=E, H=H, I=I, seed=42,
                  tokens=1, bf16=False), x, gw, ex, k)
    rb = gi.round_bf16
    for (E, H, I, k, B) in BF16_BATCHED:
        x, gw, ex = gi.reference_batched_inputs(E, H, I, B, 42)
        x, gw = rb(x), rb(gw)
        ex = tuple([rb(t) for t in lst] for lst in ex)
        emit(f"bf16_batched_E{E}_H{H}_I{I}_k{k}_B{B}",
             dict(kind="batched", gen="reference_batched_inputs", E=E, H=H, I=I, seed=42,
                  tokens=B, bf16=True), x, gw, ex, k)
    E, H, I, k = DEEPSEEK
    x, gw, ex = gi.baseline_inputs(E, H, I, 0)
    x, gw = rb(x), rb(gw)
    ex = tuple([rb(t) for t in lst] for lst in ex)
    emit(f"deepseek_bf16_E{E}_H{H}_I{I}_k{k}",
         dict(kind="single", gen="baseline_inputs", E=E, H=H, I=I, seed=0, tokens=1,
              bf16=True), x, gw, ex, k)
    del ex

    arrays["index_json"] = np.frombuffer(json.dumps(index).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **arrays)
    print(f"wrote {args.out}: {len(index)} cases, "
          f"{os.path.getsize(args.out) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
