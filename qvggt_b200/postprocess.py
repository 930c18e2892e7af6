"""Camera / geometry post-processing on the GPU (QVGGT's ``qvggt/common``).

Same names and argument meaning as the reference's
``pose_enc.pose_encoding_to_extri_intri`` (``pose_enc.py:7-65``) and
``geometry.unproject_depth_map_to_point_map`` (``geometry.py:43-96``); both
run the sm_100a kernels of ``libqvggt_b200.so`` on the current stream of the
tensors' device.  Differences: inputs must be CUDA tensors (numpy or CPU
tensors raise -- there is no CPU path), and the point map comes back as a
CUDA fp32 tensor instead of a numpy float64 array (the reference promotes to
float64 on the host; the kernels agree with it to fp32 rounding).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib


def _cuda_f32(name, t):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name}: expects CUDA tensors (no CPU path)")
    if t.dtype != torch.float32:
        raise TypeError(f"{name}: expects float32, got {t.dtype}")
    return t.contiguous()


def _stream(t):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def pose_encoding_to_extri_intri(pose_encoding: torch.Tensor, image_size_hw=None,
                                 pose_encoding_type: str = "absT_quaR_FoV", build_intrinsics: bool = True):
    """pose_encoding [..., 9] -> (extrinsics [..., 3, 4], intrinsics [..., 3, 3] or None)."""
    name = "pose_encoding_to_extri_intri"
    if pose_encoding_type != "absT_quaR_FoV":
        raise NotImplementedError
    pe = _cuda_f32(name, pose_encoding)
    if pe.shape[-1] != 9:
        raise ValueError(f"{name}: the last dimension must be 9, got {tuple(pe.shape)}")
    lead = pe.shape[:-1]
    n = pe.numel() // 9
    ext = torch.empty(*lead, 3, 4, dtype=torch.float32, device=pe.device)
    intr = None
    h = w = 0
    if build_intrinsics:
        h, w = (int(v) for v in image_size_hw)
        intr = torch.empty(*lead, 3, 3, dtype=torch.float32, device=pe.device)
    with torch.cuda.device(pe.device):
        _lib.call("qvggt_pose_encoding_to_extri_intri", C.c_void_p(pe.data_ptr()), n, h, w,
                  C.c_void_p(ext.data_ptr()), None if intr is None else C.c_void_p(intr.data_ptr()), _stream(pe))
    return ext, intr


def unproject_depth_map_to_point_map(depth_map: torch.Tensor, extrinsics_cam: torch.Tensor,
                                     intrinsics_cam: torch.Tensor) -> torch.Tensor:
    """depth_map [S, H, W] or [S, H, W, 1], extrinsics [S, 3, 4], intrinsics
    [S, 3, 3] -> world points [S, H, W, 3] (CUDA fp32)."""
    name = "unproject_depth_map_to_point_map"
    d = _cuda_f32(name, depth_map)
    if d.dim() == 4 and d.shape[-1] == 1:
        d = d[..., 0].contiguous()
    if d.dim() != 3:
        raise ValueError(f"{name}: depth must be [S, H, W(, 1)], got {tuple(depth_map.shape)}")
    S, H, W = d.shape
    e = _cuda_f32(name, extrinsics_cam)
    k = _cuda_f32(name, intrinsics_cam)
    if tuple(e.shape) != (S, 3, 4) or tuple(k.shape) != (S, 3, 3):
        raise ValueError(f"{name}: extrinsics {tuple(e.shape)} / intrinsics {tuple(k.shape)} must be [S, 3, 4] / "
                         f"[S, 3, 3] for S={S}")
    if d.device != e.device or d.device != k.device:
        raise ValueError(f"{name}: tensors on different devices")
    out = torch.empty(S, H, W, 3, dtype=torch.float32, device=d.device)
    with torch.cuda.device(d.device):
        _lib.call("qvggt_unproject_depth", C.c_void_p(d.data_ptr()), S, H, W, C.c_void_p(e.data_ptr()),
                  C.c_void_p(k.data_ptr()), C.c_void_p(out.data_ptr()), _stream(d))
    return out
