"""CPU: the post-processing oracle against golden vectors made by running the
reference's own ``pose_encoding_to_extri_intri`` and
``unproject_depth_map_to_point_map`` (``tests/golden/make_postproc_golden.py``)."""
import os

import numpy as np

from oracle import postproc as op

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "postproc_golden.npz")


def test_pose_encoding_matches_reference():
    g = np.load(GOLD)
    ext, intr = op.pose_to_extri_intri(g["pose_enc"], tuple(g["image_hw"]))
    assert np.allclose(ext, g["extrinsics"], rtol=1e-6, atol=1e-6)
    assert np.allclose(intr, g["intrinsics"], rtol=1e-6, atol=1e-4)


def test_unprojection_matches_reference():
    g = np.load(GOLD)
    pts = op.unproject_depth(g["depth"], g["extrinsics"][0, :4], g["intrinsics"][0, :4])
    assert pts.shape == g["world_points"].shape
    assert np.allclose(pts, g["world_points"], rtol=1e-6, atol=1e-5)
