"""Oracle: AWQ W4A16 packing, dequantisation, linear and GEMV (CPU).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Reference: DDsacu/QVGGT ``qvggt/runtime/awq/qmodule.py`` and
``qvggt/runtime/awq_inference_engine/csrc/quantization_new/``.
"""
from __future__ import annotations

import numpy as np
import torch


def make_divisible(c: int, divisor: int) -> int:
    """Ceil-divide (``qmodule.py:9-10``; note: returns the quotient)."""
    return (c + divisor - 1) // divisor


def calculate_zeros_width(in_features: int, group_size: int = 128, pack_num: int = 8) -> int:
    """Number of 8-group blocks of the padded scale table (``qmodule.py:13-41``)."""
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
        raise NotImplementedError(group_size)
    base_width = make_divisible(in_features // group_size, pack_num)
    return make_divisible(base_width, size_multiplier) * size_multiplier


def packed_k_index(c: int, w: int, j: int) -> int:
    """k offset of nibble ``j`` of word ``w`` of a 64-wide k-chunk ``c``.

    Layout of ``pack_intweight(interleave=4, kstride=64)`` (``qmodule.py:43-99``):
    word ``qweight[g, 64c + 16i + w]`` holds, in bits ``4j..4j+3``, the 4-bit
    value of output channel ``4g + i`` at ``k = 64c + 32*(w//8) + w%8 + 8j``.
    """
    return 64 * c + 32 * (w // 8) + (w % 8) + 8 * j


def _index_tables(K: int):
    """(word_column, nibble) for every k of one channel-in-group ``i = 0``."""
    w = np.arange(16)
    j = np.arange(4)
    c = np.arange(K // 64)
    # k[c, w, j]
    k = 64 * c[:, None, None] + 32 * (w[None, :, None] // 8) + (w[None, :, None] % 8) + 8 * j[None, None, :]
    col = 64 * c[:, None, None] + w[None, :, None] + 0 * j[None, None, :]
    return k.reshape(-1), col.reshape(-1), np.broadcast_to(j, (K // 64, 16, 4)).reshape(-1)


def pack_intweight(intweight: np.ndarray) -> np.ndarray:
    """Pack int values in 0..15 of shape [N, K] to int16 [N/4, K].

    Restates ``qmodule.py:43-99`` as an explicit scatter over the word layout of
    :func:`packed_k_index` (the reference expresses it as a chain of reshapes
    and transposes).
    """
    q = np.asarray(intweight).astype(np.int64)
    N, K = q.shape
    assert N % 4 == 0 and K % 64 == 0
    k, col, j = _index_tables(K)
    out = np.zeros((N // 4, K), dtype=np.int64)
    for i in range(4):
        vals = q[i::4][:, k]                       # [N/4, K] values in word order
        # The reference ORs the shifted values without masking (qmodule.py:88-93)
        # and truncates to int16; out-of-range values bleed exactly as there.
        np.bitwise_or.at(out, (slice(None), 16 * i + col), vals << (4 * j))
    return (out & 0xFFFF).astype(np.uint16).view(np.int16)


def unpack_intweight(qweight: np.ndarray) -> np.ndarray:
    """Inverse of :func:`pack_intweight`: int16 [N/4, K] -> int32 [N, K] in 0..15."""
    w16 = np.asarray(qweight).view(np.uint16).astype(np.int64)
    G4, K = w16.shape
    k, col, j = _index_tables(K)
    out = np.zeros((G4 * 4, K), dtype=np.int32)
    for i in range(4):
        vals = (w16[:, 16 * i + col] >> (4 * j)) & 15   # [N/4, K] in (c, w, j) order
        out[i::4][:, k] = vals
    return out


def quantize_from_linear(weight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                         group_size: int):
    """Restatement of ``WQLinear.from_linear`` (``qmodule.py:227-329``).

    weight [N, K] fp16, scales [N, K/G] fp16, zeros [N, K/G] (integers 0..15).
    Returns (qweight int16 [N/4, K], scales_t fp16 [Gpad, N], scaled_zeros_t fp16 [Gpad, N]).
    The intweight is ``round((W + z*s) / s)`` in the weight dtype (no clamp),
    computed per input column as the reference does (``qmodule.py:289-309``).
    """
    N, K = weight.shape
    G = group_size if group_size != -1 else K
    dtype = scales.dtype
    gpad = calculate_zeros_width(K, group_size) * 8
    qscales = torch.zeros((N, gpad), dtype=dtype)
    qscales[:, : scales.shape[1]] = scales
    scale_zeros = zeros * scales
    gidx = torch.arange(K) // G
    intw = torch.round((weight + scale_zeros[:, gidx]) / qscales[:, gidx]).to(torch.int32)
    qweight = pack_intweight(intw.numpy())
    szt = torch.zeros_like(qscales)
    szt[:, : scales.shape[1]] = -(qscales[:, : scales.shape[1]] * zeros.to(torch.float32)).to(dtype)
    return (torch.from_numpy(qweight), qscales.t().contiguous(), szt.t().contiguous())


def dequantize(qweight, scales_t, szeros_t, group_size: int, K: int | None = None) -> np.ndarray:
    """Bit-exact fp16 dequantised weight [N, K].

    ``dequantize_s4_to_fp16x2`` (``quantization_new/dequantize.cuh:9-51``) turns
    each nibble into the exact fp16 integer q; the kernels then apply
    ``__hfma2(q, s, sz)`` (``gemm/gemm_cuda.cu:301-307``, ``gemv/gemv_cuda.cu:126-129``):
    one fused multiply-add rounded once to fp16.  q*s + sz is exact in float64,
    so rounding that once to fp16 reproduces the fused operation.
    """
    q = unpack_intweight(np.asarray(qweight))
    N, Kq = q.shape
    K = Kq if K is None else K
    G = group_size if group_size != -1 else K
    s = np.asarray(scales_t, dtype=np.float16).astype(np.float64)      # [Gpad, N]
    z = np.asarray(szeros_t, dtype=np.float16).astype(np.float64)
    g = np.arange(K) // G
    w = q.astype(np.float64) * s[g, :].T + z[g, :].T
    return w.astype(np.float16)


def bf16_round(x) -> np.ndarray:
    """Round float64 values to bf16 (round to nearest even), once; returned as
    float32 (every bf16 is a float32).  The float64 significand is rounded to
    bf16's 8 bits directly, so no double rounding through float32.  Normal
    bf16 range only (|x| >= 2^-126 or 0), which the tests' data stay in."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float64))
    nz = x[x != 0]
    assert nz.size == 0 or np.abs(nz).min() >= 2.0 ** -126, "bf16 subnormal range not restated"
    b = x.view(np.uint64)
    lsb = (b >> np.uint64(45)) & np.uint64(1)
    r = (b + np.uint64((1 << 44) - 1) + lsb) & ~np.uint64((1 << 45) - 1)
    return r.view(np.float64).astype(np.float32)


def bf16_bits(x) -> np.ndarray:
    """uint16 bit patterns of bf16-representable float32 values."""
    return (np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b) -> np.ndarray:
    return (np.asarray(b).astype(np.uint16).astype(np.uint32) << 16).view(np.float32)


def dequantize_bf16(qweight, scales_t, szeros_t, group_size: int, K: int | None = None) -> np.ndarray:
    """Bit-exact bf16 dequantised weight [N, K] (as float32 values).

    The bf16 form of ``dequantize_s4_to_fp16x2`` (``dequantize.cuh:53-90``)
    gives the exact bf16 integer q (128 + q minus 128), and the kernels apply
    ``__hfma2(q, s, sz)`` on ``nv_bfloat162`` (``gemm/gemm_cuda.cu:906-915``,
    ``gemv/gemv_cuda.cu:130-133``): one fused multiply-add rounded once to
    bf16.  scales_t / szeros_t hold bf16 values (float32 arrays or bf16
    tensors); q*s + sz is exact in float64.
    """
    q = unpack_intweight(np.asarray(qweight))
    N, Kq = q.shape
    K = Kq if K is None else K
    G = group_size if group_size != -1 else K
    as64 = lambda t: (t.float().numpy() if isinstance(t, torch.Tensor) else np.asarray(t, np.float32)).astype(np.float64)
    s, z = as64(scales_t), as64(szeros_t)
    g = np.arange(K) // G
    return bf16_round(q.astype(np.float64) * s[g, :].T + z[g, :].T)


def w4a16_linear_bf16(x, qweight, scales_t, szeros_t, group_size: int = 128, bias=None) -> np.ndarray:
    """float64-accumulated y = x . deq_bf16(W)^T (+ bf16(y) + bias when a bias
    is given, the order of the kernels' epilogue), float64 [.., N].  x, the
    scales and the bias hold bf16 values."""
    xa = (x.float().numpy() if isinstance(x, torch.Tensor) else np.asarray(x, np.float32)).astype(np.float64)
    K = xa.shape[-1]
    w = dequantize_bf16(qweight, scales_t, szeros_t, group_size, K).astype(np.float64)
    y = xa.reshape(-1, K) @ w.T
    if bias is not None:
        b = (bias.float().numpy() if isinstance(bias, torch.Tensor) else np.asarray(bias, np.float32))
        y = bf16_round(y).astype(np.float64) + b.astype(np.float64)
    return y.reshape(*xa.shape[:-1], w.shape[0])


def make_quantized_linear_bf16(N: int, K: int, group_size: int = 128, seed: int = 0, bias: bool = True):
    """:func:`make_quantized_linear` with bf16 scales, scaled zeros and bias
    (float32 arrays of bf16 values), the way the reference's ``from_linear``
    builds them for a bf16 model: scaled zeros = bf16(-(s * z)) with s in bf16
    (``qmodule.py:302-306``)."""
    G = group_size if group_size != -1 else K
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 16, size=(N, K), dtype=np.int32)
    zeros = rng.integers(0, 16, size=(N, K // G)).astype(np.float64)
    scales = bf16_round(np.maximum(np.abs(rng.standard_normal((N, K // G))) * 0.02, 1e-4))
    gpad = calculate_zeros_width(K, group_size) * 8
    st = np.zeros((gpad, N), dtype=np.float32)
    st[: K // G] = scales.T
    szt = np.zeros((gpad, N), dtype=np.float32)
    szt[: K // G] = bf16_round(-(scales.astype(np.float64) * zeros)).T
    b = bf16_round(rng.standard_normal(N) * 0.01) if bias else None
    return dict(qweight=pack_intweight(q), scales=st, scaled_zeros=szt, bias=b, q=q, zeros=zeros,
                scales_ng=scales, group_size=group_size)


def _f16(x):
    return x.to(torch.float16) if isinstance(x, torch.Tensor) else torch.from_numpy(np.asarray(x, dtype=np.float16))


def w4a16_linear(x, qweight, scales_t, szeros_t, group_size: int = 128, bias=None) -> torch.Tensor:
    """fp32-accumulated y = x . deq(W)^T (+ bias), returned in float32.

    The oracle accumulates in fp32 (the reference's fp16 GEMM accumulates in
    fp16, ``gemm_cuda.cu:924``; the fp32 result is the more accurate one).
    """
    x = _f16(x)
    K = x.shape[-1]
    w = torch.from_numpy(dequantize(qweight, scales_t, szeros_t, group_size, K)).float()
    y = x.reshape(-1, K).float() @ w.t()
    if bias is not None:
        y = y + _f16(bias).float()
    return y.reshape(*x.shape[:-1], w.shape[0])


def wqlinear_forward_fp16(x, qweight, scales_t, szeros_t, group_size: int = 128, bias=None) -> torch.Tensor:
    """fp16 result of ``WQLinear.forward`` (``qmodule.py:333-369``).

    The GEMM/GEMV output is rounded to fp16, then ``out + bias`` is a separate
    fp16 add (one more rounding).
    """
    y = w4a16_linear(x, qweight, scales_t, szeros_t, group_size).to(torch.float16)
    if bias is not None:
        y = (y.float() + _f16(bias).float()).to(torch.float16)
    return y


def make_quantized_linear(N: int, K: int, group_size: int = 128, seed: int = 0, bias: bool = True):
    """Seeded synthetic W4A16 linear in the form BASELINE config 0 names.

    int4 q ~ U{0..15}, zeros ~ U{0..15}, scales = |N(0,1)| * 0.02 (fp16), bias ~ N(0, 0.01).
    Returns dict(qweight, scales, scaled_zeros, bias, q, zeros, scales_ng).
    """
    G = group_size if group_size != -1 else K
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 16, size=(N, K), dtype=np.int32)
    zeros = rng.integers(0, 16, size=(N, K // G)).astype(np.float32)
    scales = (np.abs(rng.standard_normal((N, K // G))) * 0.02).astype(np.float16)
    scales = np.maximum(scales, np.float16(1e-4))
    gpad = calculate_zeros_width(K, group_size) * 8
    st = np.zeros((gpad, N), dtype=np.float16)
    st[: K // G] = scales.T
    szt = np.zeros((gpad, N), dtype=np.float16)
    szt[: K // G] = (-(scales.astype(np.float32) * zeros)).astype(np.float16).T
    b = (rng.standard_normal(N) * 0.01).astype(np.float16) if bias else None
    return dict(qweight=pack_intweight(q), scales=st, scaled_zeros=szt, bias=b, q=q,
                zeros=zeros, scales_ng=scales, group_size=group_size)


def max_abs_rel(y, y_ref) -> float:
    """max|y - y_ref| / max|y_ref| (the per-linear parity metric)."""
    y = torch.as_tensor(y).double()
    y_ref = torch.as_tensor(y_ref).double()
    return float((y - y_ref).abs().max() / y_ref.abs().max().clamp_min(1e-30))


def rel_l2(y, y_ref) -> float:
    y = torch.as_tensor(y).double()
    y_ref = torch.as_tensor(y_ref).double()
    return float((y - y_ref).norm() / y_ref.norm().clamp_min(1e-30))
