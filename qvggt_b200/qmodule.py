"""Drop-in ``WQLinear`` and packing helpers (reference: ``qvggt/runtime/awq/qmodule.py``).

Same constructor, buffer names / shapes / dtypes (``qweight`` int16
[N/4, K], ``scales`` and ``scaled_zeros`` fp16 [Gpad, N], ``bias`` [N]),
``from_linear`` and ``forward`` contract as the reference, so ``model-v2.pt``
state dicts load unchanged.  ``forward`` runs the sm_100a kernels:
the GEMV kernel for up to 16 rows, the tcgen05 GEMM otherwise, with the bias
add fused into the kernel epilogue (same two fp16 roundings as the
reference's GEMM-then-add).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import awq_inference_engine as engine


def make_divisible(c, divisor):
    """Ceil-divide (reference ``qmodule.py:9-10``)."""
    return (c + divisor - 1) // divisor


def calculate_zeros_width(in_features, group_size=128, pack_num=8):
    """Padded number of 8-group blocks of the scale table (reference ``qmodule.py:13-41``)."""
    if group_size == -1:
        group_size = in_features
        size_multiplier = 1
    elif group_size >= 128:
        size_multiplier = 1
    elif group_size == 64:
        size_multiplier = 2
    elif group_size == 32:
        size_multiplier = 4
    else:
        raise NotImplementedError
    base_width = make_divisible(in_features // group_size, pack_num)
    return make_divisible(base_width, size_multiplier) * size_multiplier


def pack_intweight(unpacked_qweight: torch.Tensor, interleave: int = 4, kstride: int = 64) -> torch.Tensor:
    """Pack int values [N, K] into the int16 [N/4, K] layout of the reference
    (``qmodule.py:43-99``), on the tensor's own device.

    Word ``64c + 16i + w`` of packed row ``g`` holds in bits 4j..4j+3 the value of
    channel ``4g + i`` at ``k = 64c + 32*(w//8) + w%8 + 8j``.  Values are OR-ed
    unmasked and truncated to 16 bits, as the reference does.
    """
    if interleave != 4 or kstride != 64:
        raise NotImplementedError("only interleave=4, kstride=64")
    q = unpacked_qweight.to(torch.int32)
    N, K = q.shape
    assert N % 4 == 0 and K % 64 == 0
    # k = 64c + 32hw + 8j + wl  ->  dims (g, i, c, hw, j, wl)
    v = q.reshape(N // 4, 4, K // 64, 2, 4, 8).permute(0, 2, 1, 3, 5, 4)  # (g, c, i, hw, wl, j)
    word = v[..., 0] | (v[..., 1] << 4) | (v[..., 2] << 8) | (v[..., 3] << 12)
    word = word.reshape(N // 4, K) & 0xFFFF
    word = torch.where(word >= 0x8000, word - 0x10000, word)
    return word.to(torch.int16).contiguous()


class WQLinear(nn.Module):
    def __init__(self, w_bit, group_size, in_features, out_features, bias, dev, dtype=torch.float16):
        super().__init__()
        if w_bit not in [4]:
            raise NotImplementedError("Only 4-bit are supported for now.")
        self.in_features = in_features
        self.out_features = out_features
        self.w_bit = w_bit
        self.group_size = group_size if group_size != -1 else in_features
        self.split_k_iters = 8
        self.interleave = 4
        assert self.in_features % self.group_size == 0
        assert out_features % (32 // self.w_bit) == 0
        pack_num = 32 // self.w_bit
        int16_pack_num = 16 // self.w_bit
        assert out_features % self.interleave == 0
        gpad = calculate_zeros_width(in_features, self.group_size) * pack_num
        self.register_buffer("qweight", torch.zeros(
            (out_features // self.interleave, in_features // int16_pack_num * self.interleave),
            dtype=torch.int16, device=dev))
        self.register_buffer("scales", torch.zeros((gpad, out_features), dtype=dtype, device=dev))
        self.register_buffer("scaled_zeros", torch.zeros((gpad, out_features), dtype=dtype, device=dev))
        if bias:
            self.register_buffer("bias", torch.zeros((out_features), dtype=dtype, device=dev))
        else:
            self.bias = None

    @classmethod
    def from_linear(cls, linear, w_bit, group_size, init_only=False, scales=None, zeros=None):
        """Quantise an ``nn.Linear`` with given per-group scales / zeros
        ([N, K/G]), as the reference's ``from_linear`` (``qmodule.py:227-329``):
        intweight = round((W + z*s) / s) per input column (no clamp)."""
        awq_linear = cls(w_bit, group_size, linear.in_features, linear.out_features, linear.bias is not None,
                         linear.weight.device, dtype=linear.weight.data.dtype)
        if init_only:
            return awq_linear
        assert scales is not None and zeros is not None
        scale_zeros = zeros * scales
        dtype = scales.dtype
        G = group_size if group_size != -1 else linear.in_features
        pack_num = 32 // awq_linear.w_bit
        gpad = calculate_zeros_width(linear.in_features, group_size) * pack_num
        qscales = torch.zeros((scales.shape[0], gpad), dtype=dtype, device=scales.device)
        qscales[:, : scales.shape[1]] = scales
        awq_linear.scales = qscales.transpose(1, 0).contiguous()
        if linear.bias is not None:
            awq_linear.bias = linear.bias.detach().clone().to(dtype)
        gidx = torch.arange(linear.in_features, device=scales.device) // G
        intweight = torch.round((linear.weight.data + scale_zeros[:, gidx]) / qscales[:, gidx]).to(torch.int32)
        awq_linear.qweight = pack_intweight(intweight.contiguous(), interleave=4, kstride=64)
        zeros = zeros.to(dtype=torch.int32)
        scaled_zeros = torch.zeros_like(qscales)
        scaled_zeros[:, : scales.shape[1]] = -(qscales[:, : scales.shape[1]] * (zeros.to(torch.float32))).to(dtype)
        awq_linear.scaled_zeros = scaled_zeros.transpose(1, 0).contiguous()
        return awq_linear

    @torch.no_grad()
    def forward(self, x):
        """y = x . deq(W)^T + bias: GEMV for a few rows, the split-K small-M
        tcgen05 kernel up to 256 rows, the persistent tcgen05 GEMM beyond."""
        return engine.w4a16_linear(x.contiguous(), self.qweight, self.scales, self.scaled_zeros, self.bias,
                                   self.group_size)

    def extra_repr(self) -> str:
        return "in_features={}, out_features={}, bias={}, w_bit={}, group_size={}".format(
            self.in_features, self.out_features, self.bias is not None, self.w_bit, self.group_size)
