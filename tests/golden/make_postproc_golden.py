"""Golden vectors of the reference's camera / geometry post-processing.

Run in a container that has the reference checkout (read-only):

    python tests/golden/make_postproc_golden.py [--reference <QVGGT checkout>]

Imports ``qvggt/common/{rotation,pose_enc,geometry}.py`` from the checkout
(path from ``--reference``, else ``QVGGT_REFERENCE``, else BASELINE.json's
``reference_path``) and records, on seeded inputs:

* ``pose_encoding_to_extri_intri`` (``pose_enc.py``) on a [2, 5, 9] pose
  encoding (translations ~N(0,1), quaternions ~N(0,1) unnormalised, fields of
  view in (0.2, 2.5) rad plus the clamp edges 0 and pi) for a 294 x 518 image;
* ``unproject_depth_map_to_point_map`` (``geometry.py``) on depths [4, 21, 37, 1]
  (positive, with zeros and a negative value where the reference masks) and
  the extrinsics / intrinsics above.

Writes ``postproc_golden.npz`` next to this script.  Nothing at test time
reads the reference checkout; tests read the .npz only.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def inputs():
    """Seeded inputs (numpy), regenerated identically by the tests."""
    rng = np.random.default_rng(7)
    pe = np.zeros((2, 5, 9), np.float32)
    pe[..., :3] = rng.standard_normal((2, 5, 3))
    pe[..., 3:7] = rng.standard_normal((2, 5, 4))
    pe[..., 7:9] = rng.uniform(0.2, 2.5, (2, 5, 2))
    pe[0, 0, 7], pe[0, 1, 8] = 0.0, np.pi          # the fov clamp edges
    depth = rng.uniform(0.1, 20.0, (4, 21, 37, 1)).astype(np.float32)
    depth[0, 0, :5, 0] = 0.0
    depth[1, 3, 7, 0] = -1.0
    return pe, depth


def load_reference(ref: str):
    base = os.path.join(ref, "qvggt", "common")
    pkg = types.ModuleType("_ref_common")
    pkg.__path__ = [base]
    sys.modules["_ref_common"] = pkg
    mods = {}
    for name in ("rotation", "pose_enc", "geometry"):
        spec = importlib.util.spec_from_file_location(f"_ref_common.{name}", os.path.join(base, f"{name}.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[f"_ref_common.{name}"] = mod
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    a = ap.parse_args()
    ref = a.reference
    if ref is None:
        sys.path.insert(0, ROOT)
        from oracle.refpath import reference_path
        ref = reference_path()
    if not ref:
        raise SystemExit("reference checkout not found")
    m = load_reference(ref)
    pe, depth = inputs()
    hw = (294, 518)
    ext, intr = m["pose_enc"].pose_encoding_to_extri_intri(torch.from_numpy(pe), hw)
    pts = m["geometry"].unproject_depth_map_to_point_map(depth, ext[0, :4].numpy(), intr[0, :4].numpy())
    out = dict(pose_enc=pe, image_hw=np.array(hw), extrinsics=ext.numpy(), intrinsics=intr.numpy(), depth=depth,
               world_points=np.asarray(pts))
    path = os.path.join(HERE, "postproc_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, {k: (v.shape, v.dtype) for k, v in out.items()})


if __name__ == "__main__":
    main()
