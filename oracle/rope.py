"""Oracle: rotary position embeddings (CPU).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

* :func:`fused_rope_with_pos` restates the reference kernel
  ``csrc/rope_new/fused_rope_with_pos.cu:19-164``.
* :func:`rope2d` restates the 2-D RoPE of the VGGT aggregator (published VGGT
  algorithm, ``RotaryPositionEmbedding2D``, base frequency 100; the model code
  lives in the un-vendored ``vggt-hf`` fork): the head dimension is split in two
  halves, the first rotated by the patch row, the second by the patch column,
  each with rotate-half pairing ``i <-> i + d/4``; special tokens sit at
  position (0, 0) and patch ``p`` of a ``gw``-wide grid at ``(p // gw + 1, p % gw + 1)``.
"""
from __future__ import annotations

import numpy as np
import torch


def fused_rope_with_pos(x: torch.Tensor, freqs: torch.Tensor, transpose_output_memory: bool):
    """x [s, b, h, d] (any strides), freqs fp32 [b, s, d2] -> [s, b, h, d] in x.dtype.

    out[.., i] = x[i] cos(f_i) + r_i sin(f_i) for i < d2 with
    r_i = -x[i + d2/2] (i < d2/2) else x[i - d2/2]; angles f = freqs[b, s, i]
    (``fused_rope_with_pos.cu:29-43``); dims >= d2 are copied (``:45-56``).
    Math in fp32, one rounding to the output dtype.
    """
    s, b, hh, d = x.shape
    d2 = freqs.shape[-1]
    xf = x.float()
    f = freqs.float().permute(1, 0, 2)[:, :, None, :]           # [s, b, 1, d2]
    cos, sin = torch.cos(f), torch.sin(f)
    x1 = xf[..., :d2]
    rot = torch.cat([-x1[..., d2 // 2:], x1[..., : d2 // 2]], dim=-1)
    out = xf.clone()
    out[..., :d2] = x1 * cos + rot * sin
    out = out.to(x.dtype)
    if transpose_output_memory:
        return out.transpose(0, 1).contiguous().transpose(0, 1)
    return out.contiguous()


def rope2d_tables(max_pos: int, head_dim: int = 64, base: float = 100.0, dtype=torch.float16):
    """cos/sin tables [max_pos, head_dim/2] for one half of the head.

    As VGGT computes them for feature dim f = head_dim/2: inv_freq =
    1 / base ** (arange(0, f, 2) / f) (fp32), angles = pos * inv_freq (fp32),
    cast to the token dtype, duplicated over the two rotate-half quarters, then
    cos / sin of the cast angle, cast to the token dtype.
    """
    f = head_dim // 2
    exponents = torch.arange(0, f, 2, dtype=torch.float32) / f
    inv = 1.0 / (base ** exponents)
    p = torch.arange(max_pos, dtype=torch.float32)
    ang = torch.einsum("i,j->ij", p, inv).to(dtype)
    ang = torch.cat([ang, ang], dim=-1)
    return ang.float().cos().to(dtype), ang.float().sin().to(dtype)


def patch_positions(n_tokens: int, patch_start: int = 5, grid_w: int = 37) -> torch.Tensor:
    """[n_tokens, 2] (row, col) positions of one frame's tokens."""
    p = torch.arange(n_tokens)
    q = (p - patch_start).clamp_min(0)
    pos = torch.stack([q // grid_w + 1, q % grid_w + 1], dim=-1)
    pos[p < patch_start] = 0
    return pos


def _rope1d_f16(x: torch.Tensor, pos: torch.Tensor, cos_t, sin_t):
    """x [..., L, f] fp16, pos [L] -> fp16, rounding after each op as eager
    fp16 PyTorch does: h(h(x*cos) + h(rot(x)*sin))."""
    f = x.shape[-1]
    cos = cos_t[pos]
    sin = sin_t[pos]
    rot = torch.cat([-x[..., f // 2:], x[..., : f // 2]], dim=-1)
    a = (x.float() * cos.float()).to(torch.float16)
    b = (rot.float() * sin.float()).to(torch.float16)
    return (a.float() + b.float()).to(torch.float16)


def rope2d(x: torch.Tensor, pos: torch.Tensor, base: float = 100.0) -> torch.Tensor:
    """x [..., L, D] fp16 (D = head_dim), pos [L, 2] int -> fp16 [..., L, D]."""
    D = x.shape[-1]
    cos_t, sin_t = rope2d_tables(int(pos.max()) + 1, D, base)
    y = _rope1d_f16(x[..., : D // 2], pos[:, 0], cos_t, sin_t)
    xx = _rope1d_f16(x[..., D // 2:], pos[:, 1], cos_t, sin_t)
    return torch.cat([y, xx], dim=-1)
