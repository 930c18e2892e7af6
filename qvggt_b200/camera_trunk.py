"""The quantised trunk of VGGT's camera head on the sm_100a kernels.

QVGGT quantises, besides the aggregator, the camera head's trunk linears
(``loader.py:338-344``: every ``camera_head.*trunk.*`` linear except norms
becomes a ``WQLinear``).  The trunk is a stack of pre-LN transformer blocks
of width 2048 (16 heads x 128, no RoPE, LayerScale, exact-erf GELU MLP of
width 8192) over the camera tokens of the frames, one token per frame — so
every linear sees M = batches x S rows, the small-M regime of
``gemm_w4a16_T1`` / the GEMV in the reference (``gemm_cuda.cu:1154-1205``).

Here each linear runs on the split-K small-M tcgen05 kernel (GEMV for a few
rows), with the GELU / LayerScale-residual epilogues fused, and attention on
``attention_small`` (head_dim 128, L <= 256).  The rest of the camera head
(adaLN modulation, pose embedding, iterative refinement, pose branch) lives in
vggt-hf, which is not vendored; it is not rebuilt.
"""
from __future__ import annotations

import torch

from . import awq_inference_engine as eng
from .aggregator import Block, Linear

DIM = 2048
HEADS = 16
HEAD_DIM = 128


class CameraTrunk:
    """``depth`` trunk blocks over camera tokens [B, S, 2048] fp16."""

    def __init__(self, blocks: list[Block], heads: int = HEADS, eps: float = 1e-6):
        self.blocks = blocks
        self.heads = heads
        self.eps = eps

    def block(self, x: torch.Tensor, blk: Block, batches: int, L: int) -> None:
        """One trunk block, in place on x [batches*L, C]."""
        C = x.shape[1]
        h = eng.layernorm(x, blk.norm1_w, blk.norm1_b, self.eps)
        qkv = blk.qkv(h)                                            # [B*L, 3C] = [q | k | v]
        o = eng.attention_small(qkv[:, :C], qkv, self.heads, batches, L, k_col0=C, v_col0=2 * C)
        blk.proj(o, residual=x, gamma=blk.ls1)                      # x += half(proj(o) * ls1)
        h2 = eng.layernorm(x, blk.norm2_w, blk.norm2_b, self.eps)
        f = blk.fc1(h2, act="gelu")
        blk.fc2(f, residual=x, gamma=blk.ls2)

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """tokens [B, S, 2048] fp16 on the GPU -> [B, S, 2048] fp16."""
        B, S, C = tokens.shape
        if C != DIM:
            raise ValueError(f"camera trunk width is {DIM}, got {C}")
        x = tokens.reshape(B * S, C).contiguous().clone()
        for blk in self.blocks:
            self.block(x, blk, B, S)
        return x.reshape(B, S, C)

    __call__ = forward


def random_camera_trunk(seed: int, device, depth: int = 4, layer_scale: float = 0.01) -> CameraTrunk:
    """Random-init trunk of the VGGT-1B camera head (W4A16 g128 linears)."""
    from .synthetic import random_linear
    g = torch.Generator(device=device).manual_seed(seed)

    def vec(n, base, scale):
        return (base + scale * torch.randn(n, generator=g, device=device)).half()

    blocks = []
    for _ in range(depth):
        blocks.append(Block(
            norm1_w=vec(DIM, 1.0, 0.1), norm1_b=vec(DIM, 0.0, 0.1),
            qkv=random_linear(DIM, 3 * DIM, g, device), proj=random_linear(DIM, DIM, g, device),
            ls1=torch.full((DIM,), layer_scale, dtype=torch.float16, device=device),
            norm2_w=vec(DIM, 1.0, 0.1), norm2_b=vec(DIM, 0.0, 0.1),
            fc1=random_linear(DIM, 4 * DIM, g, device), fc2=random_linear(4 * DIM, DIM, g, device),
            ls2=torch.full((DIM,), layer_scale, dtype=torch.float16, device=device)))
    return CameraTrunk(blocks)


__all__ = ["CameraTrunk", "random_camera_trunk", "Linear", "Block"]
