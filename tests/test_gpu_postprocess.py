"""GPU: the post-processing kernels against the reference's own outputs
(``tests/golden/postproc_golden.npz``) and, at a full-size frame set, against
the oracle restatement.  fp32 kernels vs the reference's float32 torch (poses)
and float64 numpy (points): relative 1e-5."""
import os

import numpy as np
import pytest
import torch

from oracle import postproc as op

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "postproc_golden.npz")


def test_pose_encoding_matches_reference_golden():
    from qvggt_b200.postprocess import pose_encoding_to_extri_intri
    g = np.load(GOLD)
    ext, intr = pose_encoding_to_extri_intri(torch.from_numpy(g["pose_enc"]).to(DEV), tuple(g["image_hw"]))
    assert np.allclose(ext.cpu().numpy(), g["extrinsics"], rtol=1e-5, atol=1e-6)
    assert np.allclose(intr.cpu().numpy(), g["intrinsics"], rtol=1e-5, atol=1e-4)
    e2, i2 = pose_encoding_to_extri_intri(torch.from_numpy(g["pose_enc"]).to(DEV), None, build_intrinsics=False)
    assert i2 is None and torch.equal(e2, ext)


def test_unprojection_matches_reference_golden():
    from qvggt_b200.postprocess import unproject_depth_map_to_point_map
    g = np.load(GOLD)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    pts = unproject_depth_map_to_point_map(t(g["depth"]), t(g["extrinsics"][0, :4]), t(g["intrinsics"][0, :4]))
    ref = g["world_points"]
    assert np.allclose(pts.cpu().numpy(), ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())


def test_unprojection_full_frames_matches_oracle():
    """32 frames of 518 x 518 (the benchmarked frame count), depths in (0.1, 50)."""
    from qvggt_b200.postprocess import pose_encoding_to_extri_intri, unproject_depth_map_to_point_map
    g = torch.Generator().manual_seed(3)
    S, H, W = 32, 518, 518
    pe = torch.randn(1, S, 9, generator=g)
    pe[..., 7:] = torch.rand(1, S, 2, generator=g) * 1.5 + 0.5
    depth = torch.rand(S, H, W, 1, generator=g) * 50 + 0.1
    ext, intr = pose_encoding_to_extri_intri(pe.to(DEV), (H, W))
    pts = unproject_depth_map_to_point_map(depth.to(DEV), ext[0], intr[0]).cpu().numpy()
    e_ref, k_ref = op.pose_to_extri_intri(pe.numpy(), (H, W))
    ref = op.unproject_depth(depth.numpy()[:4], e_ref[0, :4], k_ref[0, :4])
    assert np.allclose(pts[:4], ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
    assert np.isfinite(pts).all()


def test_unprojection_ragged_size_and_errors():
    """A pixel count that is not a multiple of 4 takes the scalar tail."""
    from qvggt_b200.postprocess import unproject_depth_map_to_point_map
    S, H, W = 3, 7, 5
    depth = torch.rand(S, H, W) + 0.5
    ext = torch.cat([torch.eye(3).expand(S, 3, 3), torch.randn(S, 3, 1)], -1).contiguous()
    intr = torch.tensor([[100.0, 0, 2.5], [0, 90.0, 3.5], [0, 0, 1]]).expand(S, 3, 3).contiguous()
    pts = unproject_depth_map_to_point_map(depth.to(DEV), ext.to(DEV), intr.to(DEV)).cpu().numpy()
    ref = op.unproject_depth(depth.numpy(), ext.numpy(), intr.numpy())
    assert np.allclose(pts, ref, rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError):
        unproject_depth_map_to_point_map(depth, ext, intr)            # CPU tensors: no CPU path
