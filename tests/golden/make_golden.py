"""Generate the golden fixtures in this directory from the reference's own ``reference.py``.

Run in a container where the reference checkout is present::

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

For every case below it draws seeded inputs (numpy PCG64, then rounded to bfloat16 so
that the same values are exact in bf16 and fp32), runs the reference's PyTorch
forward (``reference.py:5-20`` headwise, ``reference.py:23-39`` lowrank) in float32
on the CPU, back-propagates a seeded ``dy`` with torch autograd (as ``test.py:20-30``
does), and stores inputs and float32 results as ``<case>.npz``.

The GPU box has no reference checkout, so tests only read the committed ``.npz`` files;
this script is the record of how they were made.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, kind, dict of shape parameters, has_static, residual)
CASES = [
    ("hw_hs1_w4_static_res", "headwise", dict(B=2, T=29, D=32, H=32, W=4), True, True),
    ("hw_hs8_w4_static", "headwise", dict(B=2, T=29, D=64, H=8, W=4), True, False),
    ("hw_hs16_w2_res", "headwise", dict(B=1, T=40, D=64, H=4, W=2), False, True),
    ("hw_hs2_w3_static_res", "headwise", dict(B=2, T=17, D=16, H=8, W=3), True, True),
    ("hw_hs32_w1", "headwise", dict(B=2, T=9, D=64, H=2, W=1), False, False),
    ("hw_t_lt_w", "headwise", dict(B=1, T=2, D=16, H=16, W=4), True, True),
    ("hw_hs128_w4_static_res", "headwise", dict(B=1, T=12, D=256, H=2, W=4), True, True),
    ("lr_r15_w4_static_res", "lowrank", dict(B=2, T=29, D=32, R=15, W=4), True, True),
    ("lr_r16_w4", "lowrank", dict(B=2, T=29, D=64, R=16, W=4), False, False),
    ("lr_r31_w4_static_res", "lowrank", dict(B=1, T=24, D=32, R=31, W=4), True, True),
    ("lr_r7_w2_static", "lowrank", dict(B=1, T=20, D=32, R=7, W=2), True, False),
    ("lr_r16_w3_d48_res", "lowrank", dict(B=2, T=13, D=48, R=16, W=3), False, True),
    ("lr_t_lt_w", "lowrank", dict(B=1, T=3, D=16, R=15, W=4), True, True),
    ("lr_r63_w2_static", "lowrank", dict(B=1, T=16, D=16, R=63, W=2), True, False),
    # taps beyond 4 (the reference pads W to a power of two internally, headwise.py:226)
    ("hw_hs4_w6_static_res", "headwise", dict(B=2, T=21, D=32, H=8, W=6), True, True),
    ("lr_r15_w8_static_res", "lowrank", dict(B=2, T=25, D=32, R=15, W=8), True, True),
    ("lr_r63_w5_static", "lowrank", dict(B=1, T=18, D=16, R=63, W=5), True, False),
]


def _bf16_round(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(a).to(torch.bfloat16).float().numpy()


def _load_reference(path: str):
    spec = importlib.util.spec_from_file_location("dynconv_reference", os.path.join(path, "reference.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_case(ref, name, kind, p, has_static, residual, seed):
    rng = np.random.default_rng(seed)
    B, T, D, W = p["B"], p["T"], p["D"], p["W"]
    x = _bf16_round(rng.standard_normal((B, T, D), dtype=np.float32))
    dy = _bf16_round(rng.standard_normal((B, T, D), dtype=np.float32))
    sw = _bf16_round((rng.standard_normal((W, D), dtype=np.float32) * 0.5)) if has_static else None
    arrays = {"x": x, "dy": dy}
    if sw is not None:
        arrays["static_w"] = sw
    if kind == "headwise":
        H = p["H"]
        weight = _bf16_round(rng.standard_normal((B, T, H, W), dtype=np.float32) * 0.5)
        arrays["weight"] = weight
        leaves = [torch.from_numpy(a).clone().requires_grad_() for a in (x, weight)]
        sw_t = torch.from_numpy(sw).clone().requires_grad_() if sw is not None else None
        y = ref.headwise_dynamic_convolution_ref(leaves[0], leaves[1], sw_t, residual=residual)
        y.backward(torch.from_numpy(dy))
        arrays["y"] = y.detach().numpy()
        arrays["dx"] = leaves[0].grad.numpy()
        arrays["dweight"] = leaves[1].grad.numpy()
    else:
        R = p["R"]
        z = _bf16_round(rng.standard_normal((B, T, R), dtype=np.float32) * 0.5)
        U = _bf16_round(rng.standard_normal((R, W * D), dtype=np.float32) / np.sqrt(R))
        arrays["z"] = z
        arrays["U"] = U
        leaves = [torch.from_numpy(a).clone().requires_grad_() for a in (x, z, U)]
        sw_t = torch.from_numpy(sw).clone().requires_grad_() if sw is not None else None
        y = ref.lowrank_dynamic_convolution_ref(leaves[0], leaves[1], leaves[2], sw_t, residual=residual)
        y.backward(torch.from_numpy(dy))
        arrays["y"] = y.detach().numpy()
        arrays["dx"] = leaves[0].grad.numpy()
        arrays["dz"] = leaves[1].grad.numpy()
        arrays["dU"] = leaves[2].grad.numpy()
    if sw_t is not None:
        arrays["dstatic_w"] = sw_t.grad.numpy()
    meta = dict(name=name, kind=kind, residual=bool(residual), has_static=bool(has_static), seed=seed, **p)
    arrays["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    return meta


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout (holds reference.py)")
    args = ap.parse_args()
    ref = _load_reference(args.reference)
    torch.manual_seed(0)
    index = []
    for i, (name, kind, p, has_static, residual) in enumerate(CASES):
        index.append(make_case(ref, name, kind, p, has_static, residual, seed=1000 + i))
    with open(os.path.join(HERE, "index.json"), "w") as f:
        json.dump(index, f, indent=1)
    print(f"wrote {len(index)} golden cases to {HERE}")


if __name__ == "__main__":
    sys.exit(main())
