"""Oracle: camera / geometry post-processing of the aggregator's heads' outputs.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

* ``pose_to_extri_intri`` restates ``qvggt/common/pose_enc.py:7-65``
  (``pose_encoding_to_extri_intri``, encoding "absT_quaR_FoV") with
  ``qvggt/common/rotation.py:4-25`` (``quat_to_mat``, quaternion (x, y, z, w)):
  extrinsics [R | t], intrinsics fx = (w/2) / tan(fov_w/2), fy = (h/2) /
  tan(fov_h/2) with the fields of view clamped to [1e-6, pi - 1e-6] and the
  focal lengths to [1, 1e6], principal point (w/2, h/2); float32 as the
  reference computes it in torch.
* ``unproject_depth`` restates ``qvggt/common/geometry.py:43-96``
  (``unproject_depth_map_to_point_map``): camera coordinates
  ((u - cu) d / fu, (v - cv) d / fv, d) with fu, fv floored at 1e-6, then the
  closed-form inverse of [R | t] (world = R^T cam - R^T t).  The reference
  promotes to float64 on the way (integer pixel grid minus float32 centre,
  float64 identity it writes R^T into); so does this restatement.

Pinned to ``tests/golden/postproc_golden.npz`` (made by running the reference
functions, ``tests/golden/make_postproc_golden.py``).
"""
from __future__ import annotations

import numpy as np


def quat_to_mat(q: np.ndarray) -> np.ndarray:
    """q [..., 4] (x, y, z, w), not necessarily unit -> R [..., 3, 3] (float32)."""
    q = np.asarray(q, np.float32)
    i, j, k, r = q[..., 0], q[..., 1], q[..., 2], q[..., 3]
    two_s = np.float32(2.0) / (q * q).sum(-1)
    R = np.stack([1 - two_s * (j * j + k * k), two_s * (i * j - k * r), two_s * (i * k + j * r),
                  two_s * (i * j + k * r), 1 - two_s * (i * i + k * k), two_s * (j * k - i * r),
                  two_s * (i * k - j * r), two_s * (j * k + i * r), 1 - two_s * (i * i + j * j)], -1)
    return R.reshape(q.shape[:-1] + (3, 3)).astype(np.float32)


def pose_to_extri_intri(pose_enc: np.ndarray, image_hw) -> tuple[np.ndarray, np.ndarray]:
    """pose_enc [..., 9] -> (extrinsics [..., 3, 4], intrinsics [..., 3, 3]), float32."""
    pe = np.asarray(pose_enc, np.float32)
    h, w = image_hw
    ext = np.concatenate([quat_to_mat(pe[..., 3:7]), pe[..., :3, None]], -1)
    fov_h = np.clip(pe[..., 7], 1e-6, np.pi - 1e-6).astype(np.float32)
    fov_w = np.clip(pe[..., 8], 1e-6, np.pi - 1e-6).astype(np.float32)
    fy = np.clip(np.float32(h / 2.0) / np.tan(fov_h / np.float32(2.0)), 1.0, 1e6)
    fx = np.clip(np.float32(w / 2.0) / np.tan(fov_w / np.float32(2.0)), 1.0, 1e6)
    intr = np.zeros(pe.shape[:-1] + (3, 3), np.float32)
    intr[..., 0, 0], intr[..., 1, 1] = fx, fy
    intr[..., 0, 2], intr[..., 1, 2], intr[..., 2, 2] = w / 2, h / 2, 1.0
    return ext.astype(np.float32), intr


def unproject_depth(depth: np.ndarray, extrinsics: np.ndarray, intrinsics: np.ndarray) -> np.ndarray:
    """depth [S, H, W] or [S, H, W, 1] -> world points [S, H, W, 3] (float64)."""
    d = np.asarray(depth, np.float32)
    if d.ndim == 4:
        d = d[..., 0]
    S, H, W = d.shape
    v, u = np.meshgrid(np.arange(H), np.arange(W), indexing="ij")
    out = np.empty((S, H, W, 3), np.float64)
    for s in range(S):
        K = np.asarray(intrinsics[s], np.float32)
        E = np.asarray(extrinsics[s], np.float32)
        fu, fv = max(float(K[0, 0]), 1e-6), max(float(K[1, 1]), 1e-6)
        cam = np.stack([(u - K[0, 2]) * d[s] / fu, (v - K[1, 2]) * d[s] / fv, d[s]], -1).astype(np.float32)
        rt = E[:, :3].T.astype(np.float32)
        t_w = (-(rt @ E[:, 3:])).astype(np.float32)[:, 0]
        out[s] = cam.astype(np.float64) @ rt.T.astype(np.float64) + t_w.astype(np.float64)
    return out
