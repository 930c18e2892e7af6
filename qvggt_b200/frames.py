"""Frame sizes other than 518 x 518: the crop rule and the DINOv2 position table.

QVGGT's image loader (``qvggt/inference/io.py:50-100``, mode "crop", the
default) resizes every image to width 518 and height
``round(h * 518 / w / 14) * 14`` and centre-crops a height above 518 to 518,
so frames are 518 wide and at most 518 tall: 37 patch columns and up to 37
patch rows (mode "pad" makes them 518 x 518).  The aggregator's kernels take the
patch grid as parameters; what changes with the height is the DINOv2 front's
position table, which the checkpoint stores for 37 x 37 patches and the model
resizes to the frame's grid (the published DINOv2 ``interpolate_pos_encoding``:
the class position is kept, the patch positions are resampled as a
37 x 37 x C image with bicubic, antialiased interpolation to rows x cols).

This is one-time host set-up (per frame size); the table is then added to the
tokens by the ``assemble_tokens`` kernel.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

TARGET = 518
PATCH = 14


def crop_size(height: int, width: int, target: int = TARGET, mode: str = "crop") -> tuple[int, int, int, int]:
    """(resized height, resized width, frame height, frame width) of an image
    of ``height`` x ``width`` pixels under the loader's rule (``io.py:50-100``).
    "crop": width ``target``, height rounded to a multiple of 14 and cropped to
    ``target``; "pad": the longer side ``target``, padded to a square."""
    if height <= 0 or width <= 0:
        raise ValueError("image sides must be positive")
    if mode == "pad":
        if width >= height:
            rw, rh = target, round(height * (target / width) / PATCH) * PATCH
        else:
            rh, rw = target, round(width * (target / height) / PATCH) * PATCH
        return rh, rw, target, target
    if mode != "crop":
        raise ValueError(f"mode must be 'crop' or 'pad', not {mode!r}")
    rw = target
    rh = round(height * (target / width) / PATCH) * PATCH
    return rh, rw, min(rh, target), rw


def interpolate_position_table(pos_embed: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """DINOv2's position table for a rows x cols patch grid.

    ``pos_embed``: [1 + M*M, C] (class position, then an M x M patch grid in
    row-major order).  Returns fp32 [1 + rows*cols, C] on the CPU; the input
    itself when the grid is unchanged.  Bicubic, antialiased (the resampling
    filter widens when shrinking), computed in fp32."""
    pe = pos_embed.detach().float().cpu().reshape(-1, pos_embed.shape[-1])
    n = pe.shape[0] - 1
    M = int(round(math.sqrt(n)))
    if M * M != n:
        raise ValueError(f"the position table's {n} patch entries are not a square grid")
    if rows <= 0 or cols <= 0:
        raise ValueError("the patch grid must be at least 1 x 1")
    if (rows, cols) == (M, M):
        return pe
    C = pe.shape[1]
    grid = pe[1:].reshape(1, M, M, C).permute(0, 3, 1, 2)
    out = F.interpolate(grid, size=(rows, cols), mode="bicubic", antialias=True, align_corners=False)
    return torch.cat([pe[:1], out.permute(0, 2, 3, 1).reshape(rows * cols, C)], dim=0)


def token_position_table(pos_embed: torch.Tensor, rows: int, cols: int, n_special: int = 5) -> torch.Tensor:
    """The per-token table ``assemble_tokens`` adds to the DINOv2 sequence
    [cls | registers | patches]: the class position in row 0, zeros for the
    registers (DINOv2 gives them no position), the patch positions after them;
    fp16 [n_special + rows*cols, C] on the CPU."""
    t = interpolate_position_table(pos_embed, rows, cols)
    out = torch.zeros(n_special + rows * cols, t.shape[1], dtype=torch.float32)
    out[0] = t[0]
    out[n_special:] = t[1:]
    return out.to(torch.float16)
