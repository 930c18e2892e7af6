"""Generate golden fixtures from the reference's own Python packing code.

Run in a container that has the reference checkout (read-only):

    python tests/golden/make_golden.py --reference <path-to-QVGGT-checkout>

It imports ``qvggt/runtime/awq/qmodule.py`` (the CUDA extension it imports at
module top is replaced by an empty stub module -- only the CPU packing code is
exercised) and records, for seeded inputs:

* ``calculate_zeros_width`` over a grid of (in_features, group_size);
* ``pack_intweight(interleave=4, kstride=64)`` of seeded int matrices,
  including out-of-range values (the reference does not mask);
* ``WQLinear.from_linear`` buffers (qweight, scales, scaled_zeros, bias) for
  seeded fp32 linears, scales and zeros.

Output: ``tests/golden/awq_pack_golden.npz`` (a few hundred KB).
Nothing at test time reads the reference checkout; tests read the .npz only.
"""
from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "awq_pack_golden.npz"))
    args = ap.parse_args()

    sys.modules.setdefault("awq_inference_engine", types.ModuleType("awq_inference_engine"))
    sys.path.insert(0, os.path.join(args.reference, "qvggt", "runtime", "awq"))
    import qmodule  # noqa: E402  (reference code)

    out = {}
    czw = []
    for K in (64, 128, 256, 384, 512, 1024, 1536, 2048, 4096):
        for G in (32, 64, 128, 256, -1):
            if G != -1 and K % G:
                continue
            czw.append((K, G, qmodule.calculate_zeros_width(K, G)))
    out["czw"] = np.array(czw, dtype=np.int64)

    rng = np.random.default_rng(1234)
    for idx, (N, K, lo, hi) in enumerate([(8, 64, 0, 16), (16, 128, 0, 16), (64, 256, 0, 16),
                                         (12, 192, 0, 16), (8, 128, -3, 20)]):
        q = rng.integers(lo, hi, size=(N, K)).astype(np.int32)
        packed = qmodule.pack_intweight(torch.from_numpy(q), interleave=4, kstride=64).numpy()
        out[f"pack{idx}_in"] = q
        out[f"pack{idx}_out"] = packed

    torch.manual_seed(4321)
    for idx, (N, K, G) in enumerate([(64, 256, 128), (32, 256, 64), (16, 128, 32), (128, 1024, 128)]):
        lin = torch.nn.Linear(K, N, bias=True)
        w = lin.weight.data
        ng = K // G
        wg = w.reshape(N, ng, G)
        mx, mn = wg.amax(-1), wg.amin(-1)
        scales = ((mx - mn).clamp_min(1e-5) / 15.0)
        zeros = torch.round(-mn / scales).clamp(0, 15)
        lin = lin.half()
        scales = scales.half()
        wq = qmodule.WQLinear.from_linear(lin, 4, G, scales=scales, zeros=zeros)
        out[f"lin{idx}_weight"] = lin.weight.data.numpy()
        out[f"lin{idx}_bias"] = lin.bias.data.numpy()
        out[f"lin{idx}_scales_in"] = scales.numpy()
        out[f"lin{idx}_zeros_in"] = zeros.numpy()
        out[f"lin{idx}_G"] = np.array(G)
        out[f"lin{idx}_qweight"] = wq.qweight.detach().numpy()
        out[f"lin{idx}_scales"] = wq.scales.detach().numpy()
        out[f"lin{idx}_scaled_zeros"] = wq.scaled_zeros.detach().numpy()
        out[f"lin{idx}_out_bias"] = wq.bias.detach().numpy()
    np.savez_compressed(args.out, **out)
    print("wrote", args.out, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
