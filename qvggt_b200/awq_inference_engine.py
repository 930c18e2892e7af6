"""Drop-in replacement of the reference's ``awq_inference_engine`` extension.

Same function names, argument order, dtypes, layouts and ownership as the
bindings in ``qvggt/runtime/awq_inference_engine/csrc/pybind.cpp:18-36``; every
op runs a sm_100a kernel of ``libqvggt_b200.so`` through its C ABI on the
current PyTorch CUDA stream of the tensor's device.  There is no CPU path:
CPU tensors, wrong dtypes or unsupported shapes raise.

Ops outside the VGGT hot path (``layernorm_forward_cuda`` = T5 RMSNorm,
``rotary_embedding_neox`` = 1-D LLM RoPE, ``single_query_attention`` =
decode-time attention, ``silu_and_mul`` = SwiGLU) raise ``NotImplementedError``.

New ops of the hot path (no reference name): :func:`w4a16_linear`,
:func:`f16_linear`, :func:`layernorm`, :func:`qkv_rope2d`, :func:`attention`.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

__all__ = [
    "gemm_forward_cuda_new", "gemv_forward_cuda_new", "w8a8_gemm_forward_cuda",
    "w8a8_gemm_fuse_bias_forward_cuda", "invoke_quant", "rms_norm_general", "gelu_and_quant",
    "fused_rope_with_pos_forward_func", "w4a16_linear", "f16_linear", "layernorm", "qkv_rope2d",
    "attention", "attention_small", "i8_gemm_i32", "small_linear", "attention_ex", "attention_plan",
    "attention_scratch_bytes",
]


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


# The current stream's raw handle without building a torch.cuda.Stream object
# per call (the aggregator issues ~500 launches per forward).
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t: torch.Tensor):
    if _raw_stream is not None:
        return C.c_void_p(_raw_stream(t.device.index))
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _check_cuda(name, *ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError(f"{name}: all tensors must be CUDA tensors (no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{name}: tensors on different devices")
    return dev


def _check_dtype(name, t, *dtypes):
    if t is not None and t.dtype not in dtypes:
        raise TypeError(f"{name}: expected {dtypes}, got {t.dtype}")


def _contig(name, *ts):
    for t in ts:
        if t is not None and not t.is_contiguous():
            raise ValueError(f"{name}: tensors must be contiguous")


def _check_shape(name, cond: bool, what: str):
    if not cond:
        raise ValueError(f"{name}: {what}")


def _check_w4_weights(name, qweight, scales, scaled_zeros, K: int, group_size: int, dtype=torch.float16):
    """qweight int16 [N/4, K]; scales / scaled_zeros ``dtype`` [gpad, N] with at
    least K / group_size group rows (the kernels read that many)."""
    _check_dtype(name, qweight, torch.int16)
    _check_dtype(name, scales, dtype)
    _check_dtype(name, scaled_zeros, dtype)
    _check_shape(name, qweight.dim() == 2 and qweight.shape[1] == K,
                 f"qweight {tuple(qweight.shape)} must be [N/4, K={K}]")
    N = qweight.shape[0] * 4
    _check_shape(name, group_size > 0 and K % group_size == 0, f"K={K} is not a multiple of group_size={group_size}")
    for t, n in ((scales, "scales"), (scaled_zeros, "scaled_zeros")):
        _check_shape(name, t.dim() == 2 and t.shape[1] == N and t.shape[0] >= K // group_size,
                     f"{n} {tuple(t.shape)} must be [>= {K // group_size}, N={N}]")
    return N


def _check_epilogue(name, M: int, N: int, bias=None, residual=None, gamma=None, out=None):
    """bias / gamma fp16 with >= N entries; residual / out fp16 contiguous [.., N] with M rows."""
    for t, n in ((bias, "bias"), (gamma, "gamma")):
        if t is not None:
            _check_dtype(name, t, torch.float16)
            _check_shape(name, t.numel() >= N, f"{n} has {t.numel()} entries, needs {N}")
    for t, n in ((residual, "residual"), (out, "out")):
        if t is not None:
            _check_dtype(name, t, torch.float16)
            _contig(name, t)
            _check_shape(name, t.shape[-1] == N and t.numel() == M * N,
                         f"{n} {tuple(t.shape)} must hold {M} rows of N={N}")


def _check_rows(name, t, rows: int, cols: int, what: str):
    """A row-major fp16 operand read through its row stride: 2-D, unit column
    stride, at least `rows` rows and `cols` columns."""
    _check_dtype(name, t, torch.float16)
    _check_shape(name, t.dim() == 2 and t.stride(-1) == 1 and t.shape[0] >= rows and t.shape[1] >= cols,
                 f"{what} {tuple(t.shape)} (strides {tuple(t.stride())}) must be a row-major view with >= {rows} "
                 f"rows and >= {cols} columns")


class _Dev:
    """Makes `dev` the current CUDA device for the launch (the C ABI launches
    on the current device), restoring the previous one after; a no-op when
    it already is current."""

    def __init__(self, dev):
        self.idx = dev.index
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *a):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


# --------------------------------------------------------------------- W4A16
def gemm_forward_cuda_new(in_feats, qweight, scales, scaled_zeros, group_size: int = 128):
    """C = in_feats . deq(qweight)^T (``gemm_cuda.cu:1125-1235``).

    in_feats fp16 or bf16 [..., K]; qweight int16 [N/4, K]; scales /
    scaled_zeros [gpad, N] of the same dtype as in_feats (the reference's
    TORCH_CHECKs, ``gemm_cuda.cu:1143-1146``).  Returns a new tensor [..., N]
    of that dtype.  The reference fixes the group size at 128; it is a
    keyword here for other multiples of 64.
    """
    name = "gemm_forward_cuda_new"
    dev = _check_cuda(name, in_feats, qweight, scales, scaled_zeros)
    _check_dtype(name, in_feats, torch.float16, torch.bfloat16)
    bf16 = in_feats.dtype == torch.bfloat16
    _contig(name, in_feats, qweight, scales, scaled_zeros)
    K = in_feats.shape[-1]
    N = _check_w4_weights(name, qweight, scales, scaled_zeros, K, group_size, in_feats.dtype)
    M = in_feats.numel() // K
    out = torch.empty(*in_feats.shape[:-1], N, dtype=in_feats.dtype, device=dev)
    with _Dev(dev):
        if 1 <= M <= SMALL_M_MAX:
            _small_linear(2 if bf16 else 0, in_feats, qweight, scales, scaled_zeros, group_size, None, out, M, N, K,
                          0, None, None)
        else:
            _lib.call("qvggt_w4a16_gemm_bf16" if bf16 else "qvggt_w4a16_gemm", _ptr(in_feats), _ptr(qweight),
                      _ptr(scales), _ptr(scaled_zeros), None, _ptr(out), M, N, K, scales.shape[0], group_size,
                      _stream(in_feats))
    return out


def gemv_forward_cuda_new(in_feats, qweight, scales, scaled_zeros, m: int, n: int, k: int, group_size: int):
    """y = in_feats . deq(qweight)^T for m <= 16 rows (``gemv_cuda.cu:197-281``);
    fp16 or bf16 in_feats, with scales / scaled_zeros of the same dtype."""
    name = "gemv_forward_cuda_new"
    dev = _check_cuda(name, in_feats, qweight, scales, scaled_zeros)
    _check_dtype(name, in_feats, torch.float16, torch.bfloat16)
    _check_dtype(name, scales, in_feats.dtype)
    _check_dtype(name, scaled_zeros, in_feats.dtype)
    _contig(name, in_feats, qweight, scales, scaled_zeros)
    if not (1 <= m <= 16):
        raise RuntimeError("Unsupported batch size for gemv kernel.")
    if group_size % 32 or k % group_size:
        raise RuntimeError("Unsupported group size for gemv kernel.")
    _check_shape(name, in_feats.shape[-1] == k and in_feats.numel() >= m * k,
                 f"in_feats {tuple(in_feats.shape)} must hold m={m} rows of k={k}")
    _check_shape(name, _check_w4_weights(name, qweight, scales, scaled_zeros, k, group_size, in_feats.dtype) == n,
                 f"qweight {tuple(qweight.shape)} does not give n={n} channels")
    out = torch.empty(*in_feats.shape[:-1], n, dtype=in_feats.dtype, device=dev)
    entry = "qvggt_w4a16_gemv_bf16" if in_feats.dtype == torch.bfloat16 else "qvggt_w4a16_gemv"
    with _Dev(dev):
        _lib.call(entry, _ptr(in_feats), _ptr(qweight), _ptr(scales), _ptr(scaled_zeros), None,
                  _ptr(out), m, n, k, scales.shape[0], group_size, _stream(in_feats))
    return out


def w4a16_linear(x, qweight, scales, scaled_zeros, bias=None, group_size: int = 128, act: str | None = None,
                 residual=None, gamma=None, out=None):
    """Fused W4A16 linear: ``half(half(x.W^T) + bias)`` then optionally
    ``gelu`` (act='gelu') or an in-place LayerScale residual update
    ``residual += half(y * gamma)`` (returns ``residual``).  Up to
    ``GEMV_M_MAX`` rows (plain / bias epilogue) use the GEMV kernel, up to
    ``SMALL_M_MAX`` rows the split-K small-M kernel, more the persistent
    tcgen05 GEMM.  bf16 ``x`` (with bf16 scales, zeros, bias): the plain /
    bias linear only, ``bf16(bf16(x.W^T) + bias)``."""
    name = "w4a16_linear"
    dev = _check_cuda(name, x, qweight, scales, scaled_zeros, bias, residual, gamma, out)
    _check_dtype(name, x, torch.float16, torch.bfloat16)
    if x.dtype == torch.bfloat16:
        return _w4a16_linear_bf16(name, dev, x, qweight, scales, scaled_zeros, bias, group_size, act, residual,
                                  out)
    _contig(name, x, qweight, scales, scaled_zeros, bias, gamma)
    K = x.shape[-1]
    N = _check_w4_weights(name, qweight, scales, scaled_zeros, K, group_size)
    M = x.numel() // K
    _check_epilogue(name, M, N, bias, residual, gamma, None if residual is not None else out)
    _check_shape(name, residual is None or gamma is not None, "a residual update needs gamma")
    if residual is not None:
        out = residual
    elif out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.float16, device=dev)
    if M == 0:
        return out
    with _Dev(dev):
        if M <= GEMV_M_MAX and act is None and residual is None:
            _lib.call("qvggt_w4a16_gemv", _ptr(x), _ptr(qweight), _ptr(scales), _ptr(scaled_zeros), _ptr(bias),
                      _ptr(out), M, N, K, scales.shape[0], group_size, _stream(x))
        elif 1 <= M <= SMALL_M_MAX:
            _small_linear(0, x, qweight, scales, scaled_zeros, group_size, bias, out, M, N, K,
                          1 if act == "gelu" else 0, residual, gamma)
        else:
            _lib.call("qvggt_w4a16_linear_ex", _ptr(x), K, _ptr(qweight), _ptr(scales), _ptr(scaled_zeros),
                      _ptr(bias), _ptr(out), N, M, N, K, scales.shape[0], group_size, 1 if act == "gelu" else 0,
                      _ptr(residual), N if residual is not None else 0, _ptr(gamma), _stream(x))
    return out


def _w4a16_linear_bf16(name, dev, x, qweight, scales, scaled_zeros, bias, group_size, act, residual, out):
    """bf16 form of :func:`w4a16_linear` (the reference's bf16 instantiation of
    gemv_forward_cuda_new / gemm_forward_cuda_new plus WQLinear's bias add)."""
    if act is not None or residual is not None:
        raise NotImplementedError(f"{name}: bf16 activations take the plain / bias linear only")
    _contig(name, x, qweight, scales, scaled_zeros, bias)
    K = x.shape[-1]
    N = _check_w4_weights(name, qweight, scales, scaled_zeros, K, group_size, torch.bfloat16)
    M = x.numel() // K
    if bias is not None:
        _check_dtype(name, bias, torch.bfloat16)
        _check_shape(name, bias.numel() >= N, f"bias has {bias.numel()} entries, needs {N}")
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=dev)
    else:
        _check_dtype(name, out, torch.bfloat16)
        _contig(name, out)
        _check_shape(name, out.shape[-1] == N and out.numel() == M * N, f"out {tuple(out.shape)} must hold {M} rows of N={N}")
    if M == 0:
        return out
    with _Dev(dev):
        if M <= GEMV_M_MAX:
            _lib.call("qvggt_w4a16_gemv_bf16", _ptr(x), _ptr(qweight), _ptr(scales), _ptr(scaled_zeros), _ptr(bias),
                      _ptr(out), M, N, K, scales.shape[0], group_size, _stream(x))
        elif M <= SMALL_M_MAX:
            _small_linear(2, x, qweight, scales, scaled_zeros, group_size, bias, out, M, N, K, 0, None, None)
        else:
            _lib.call("qvggt_w4a16_gemm_bf16", _ptr(x), _ptr(qweight), _ptr(scales), _ptr(scaled_zeros), _ptr(bias),
                      _ptr(out), M, N, K, scales.shape[0], group_size, _stream(x))
    return out


def qkv_rope_linear(x, lin, heads: int, cos_tab, sin_tab, tokens_per_frame: int = 1374, patch_start: int = 5,
                    grid_w: int = 37, token_offset: int = 0, q_out=None, kv_out=None, qk_norm=None,
                    eps: float = 1e-6):
    """qkv projection (W4A16 ``lin.kind == 'w4'`` or dense fp16) with the
    split and VGGT 2-D RoPE fused into the GEMM epilogue.
    Returns (q [M, C] roped, kv [M, 2C] = [k roped | v])."""
    name = "qkv_rope_linear"
    dev = _check_cuda(name, x, lin.bias, cos_tab, sin_tab, q_out, kv_out)
    _check_dtype(name, x, torch.float16)
    _contig(name, x, cos_tab, sin_tab, q_out, kv_out)
    K = x.shape[-1]
    M = x.numel() // K
    Cd = heads * 64
    if lin.kind == "w4":
        N = _check_w4_weights(name, lin.qweight, lin.scales, lin.scaled_zeros, K, lin.group_size)
    else:
        _check_shape(name, lin.weight.dim() == 2 and lin.weight.shape[1] == K, "weight must be [3C, K]")
        N = lin.weight.shape[0]
    _check_shape(name, N == 3 * Cd, f"the qkv linear has {N} outputs, needs 3 * {Cd}")
    _check_epilogue(name, M, N, lin.bias)
    if q_out is None:
        q_out = torch.empty(M, Cd, dtype=torch.float16, device=dev)
    if kv_out is None:
        kv_out = torch.empty(M, 2 * Cd, dtype=torch.float16, device=dev)
    _check_epilogue(name, M, Cd, out=q_out)
    _check_epilogue(name, M, 2 * Cd, out=kv_out)
    qn = qk_norm if qk_norm is not None else (None, None, None, None)
    if lin.kind == "w4":
        wk, b, s, z, gpad, G = 0, lin.qweight, lin.scales, lin.scaled_zeros, lin.scales.shape[0], lin.group_size
    else:
        wk, b, s, z, gpad, G = 1, lin.weight, None, None, 0, 128
    with _Dev(dev):
        _lib.call("qvggt_qkv_rope_linear", _ptr(x), wk, _ptr(b), _ptr(s), _ptr(z), gpad, G, _ptr(lin.bias),
                  _ptr(q_out), _ptr(kv_out), M, K, Cd, token_offset, tokens_per_frame, patch_start, grid_w,
                  _ptr(cos_tab), _ptr(sin_tab), cos_tab.shape[0], 1 if qk_norm is not None else 0, _ptr(qn[0]),
                  _ptr(qn[1]), _ptr(qn[2]), _ptr(qn[3]), float(eps), _stream(x))
    return q_out, kv_out


def f16_linear(x, weight, bias=None, act: str | None = None, residual=None, gamma=None, out=None):
    """Dense fp16 linear (weight [N, K]) with the same fused epilogues."""
    name = "f16_linear"
    dev = _check_cuda(name, x, weight, bias, residual, gamma, out)
    _check_dtype(name, x, torch.float16)
    _check_dtype(name, weight, torch.float16)
    _contig(name, x, weight, bias, gamma)
    K = x.shape[-1]
    _check_shape(name, weight.dim() == 2 and weight.shape[1] == K, f"weight {tuple(weight.shape)} must be [N, K={K}]")
    N = weight.shape[0]
    M = x.numel() // K
    _check_epilogue(name, M, N, bias, residual, gamma, None if residual is not None else out)
    _check_shape(name, residual is None or gamma is not None, "a residual update needs gamma")
    if residual is not None:
        out = residual
    elif out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.float16, device=dev)
    if M == 0:
        return out
    with _Dev(dev):
        if 1 <= M <= SMALL_M_MAX:
            _small_linear(1, x, weight, None, None, 128, bias, out, M, N, K, 1 if act == "gelu" else 0,
                          residual, gamma)
        else:
            _lib.call("qvggt_f16_linear_ex", _ptr(x), K, _ptr(weight), _ptr(bias), _ptr(out), N, M, N, K,
                      1 if act == "gelu" else 0, _ptr(residual), N if residual is not None else 0, _ptr(gamma),
                      _stream(x))
    return out


# ------------------------------------------------------------------- small M
# Row counts routed to the split-K small-M kernel (qvggt_small_linear); up to
# GEMV_M_MAX rows without a fused activation/residual use the GEMV.  Measured
# on B200 at the camera-trunk shapes (dim 2048, one row per frame).
SMALL_M_MAX = 256
GEMV_M_MAX = 4


def _small_linear(kind, x, w, scales, zeros, group_size, bias, out, M, N, K, act, residual, gamma):
    _lib.call("qvggt_small_linear", kind, _ptr(x), K, _ptr(w), _ptr(scales), _ptr(zeros),
              scales.shape[0] if scales is not None else 0, group_size, _ptr(bias), _ptr(out), N, M, N, K, act,
              _ptr(residual), N if residual is not None else 0, _ptr(gamma), _stream(x))


def small_linear_plan(weight_kind: int, M: int, N: int, K: int) -> dict:
    """Launch plan of :func:`small_linear` on the current device."""
    info = (C.c_int32 * 5)()
    _lib.call("qvggt_small_linear_plan", weight_kind, M, N, K, info)
    return dict(rows=info[0], splits=info[1], kb_per_cta=info[2], ctas=info[3], active_clusters=info[4])


def small_linear(x, weight, scales=None, scaled_zeros=None, bias=None, group_size: int = 128,
                 act: str | None = None, residual=None, gamma=None, out=None):
    """Linear for 1..256 rows on the split-K small-M kernel (always, whatever
    ``SMALL_M_MAX`` says): W4A16 when
    ``scales`` is given (``weight`` = qweight int16 [N/4, K]), else dense fp16
    ``weight`` [N, K].  Same epilogues and rounding as :func:`w4a16_linear`."""
    name = "small_linear"
    dev = _check_cuda(name, x, weight, scales, scaled_zeros, bias, residual, gamma, out)
    _check_dtype(name, x, torch.float16)
    _contig(name, x, weight, scales, scaled_zeros, bias, gamma)
    kind = 0 if scales is not None else 1
    K = x.shape[-1]
    if kind == 0:
        N = _check_w4_weights(name, weight, scales, scaled_zeros, K, group_size)
    else:
        _check_dtype(name, weight, torch.float16)
        _check_shape(name, weight.dim() == 2 and weight.shape[1] == K,
                     f"weight {tuple(weight.shape)} must be [N, K={K}]")
        N = weight.shape[0]
    M = x.numel() // K
    _check_epilogue(name, M, N, bias, residual, gamma, None if residual is not None else out)
    if residual is not None:
        out = residual
    elif out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.float16, device=dev)
    with _Dev(dev):
        _small_linear(kind, x, weight, scales, scaled_zeros, group_size, bias, out, M, N, K,
                      1 if act == "gelu" else 0, residual, gamma)
    return out


# ---------------------------------------------------------------------- W8A8
def _w8a8(name, in_feats, kernel, wscales, ascales, out, bias):
    dev = _check_cuda(name, in_feats, kernel, wscales, ascales, out, bias)
    _check_dtype(name, in_feats, torch.int8)
    _check_dtype(name, kernel, torch.int8)
    _check_dtype(name, out, torch.float16)
    _check_dtype(name, wscales, torch.float16)
    _check_dtype(name, ascales, torch.float16)
    _check_dtype(name, bias, torch.float16)
    _contig(name, in_feats, kernel, wscales, ascales, out, bias)
    _check_shape(name, in_feats.dim() == 2, f"in_feats {tuple(in_feats.shape)} must be [M, K]")
    M, K = in_feats.shape[0], in_feats.shape[1]
    N = out.shape[-1]
    _check_shape(name, tuple(kernel.shape) == (N, K), f"kernel {tuple(kernel.shape)} must be [N={N}, K={K}]")
    _check_shape(name, out.numel() == M * N, f"out {tuple(out.shape)} must be [M={M}, N={N}]")
    _check_shape(name, wscales.numel() >= N, f"wscales has {wscales.numel()} entries, needs N={N}")
    _check_shape(name, ascales.numel() >= M, f"ascales has {ascales.numel()} entries, needs M={M}")
    _check_shape(name, bias is None or bias.numel() >= N, f"bias needs N={N} entries")
    with _Dev(dev):
        _lib.call("qvggt_w8a8_gemm", _ptr(in_feats), _ptr(kernel), _ptr(wscales), _ptr(ascales), _ptr(bias),
                  _ptr(out), M, N, K, _stream(in_feats))


def w8a8_gemm_forward_cuda(in_feats, kernel, wscales, ascales, out_feats):
    """out = half(float(acc) * (ws * as)) (``w8a8_gemm_cuda.cu:881-922``); writes out_feats."""
    _w8a8("w8a8_gemm_forward_cuda", in_feats, kernel, wscales, ascales, out_feats, None)


def w8a8_gemm_fuse_bias_forward_cuda(in_feats, kernel, wscales, ascales, out_feats, bias):
    """out = half(fma(acc * ws, as, bias)) (``w8a8_gemm_cuda.cu:564-607``); writes out_feats."""
    _w8a8("w8a8_gemm_fuse_bias_forward_cuda", in_feats, kernel, wscales, ascales, out_feats, bias)


def w8a8_gemm_residual(in_feats, kernel, wscales, ascales, bias, gamma, residual):
    """residual += half(half(W8A8 GEMM(+bias)) * gamma) (LayerScale residual fused)."""
    name = "w8a8_gemm_residual"
    dev = _check_cuda(name, in_feats, kernel, wscales, ascales, bias, gamma, residual)
    _check_dtype(name, in_feats, torch.int8)
    _check_dtype(name, kernel, torch.int8)
    _check_dtype(name, wscales, torch.float16)
    _check_dtype(name, ascales, torch.float16)
    _contig(name, in_feats, kernel, wscales, ascales, bias, gamma, residual)
    _check_shape(name, in_feats.dim() == 2 and kernel.dim() == 2 and kernel.shape[1] == in_feats.shape[1],
                 f"in_feats {tuple(in_feats.shape)} / kernel {tuple(kernel.shape)} must be [M, K] / [N, K]")
    M, K = in_feats.shape[0], in_feats.shape[1]
    N = kernel.shape[0]
    _check_shape(name, wscales.numel() >= N, f"wscales has {wscales.numel()} entries, needs N={N}")
    _check_shape(name, ascales.numel() >= M, f"ascales has {ascales.numel()} entries, needs M={M}")
    _check_shape(name, gamma is not None, "gamma is required")
    _check_epilogue(name, M, N, bias, residual, gamma)
    with _Dev(dev):
        _lib.call("qvggt_w8a8_gemm_residual", _ptr(in_feats), _ptr(kernel), _ptr(wscales), _ptr(ascales), _ptr(bias),
                  _ptr(gamma), _ptr(residual), M, N, K, _stream(in_feats))
    return residual


def i8_gemm_i32(in_feats, kernel):
    """Raw int32 accumulators of the int8 GEMM (for bit-exact checks)."""
    name = "i8_gemm_i32"
    dev = _check_cuda(name, in_feats, kernel)
    _check_dtype(name, in_feats, torch.int8)
    _check_dtype(name, kernel, torch.int8)
    _contig(name, in_feats, kernel)
    _check_shape(name, in_feats.dim() == 2 and kernel.dim() == 2 and kernel.shape[1] == in_feats.shape[1],
                 f"in_feats {tuple(in_feats.shape)} / kernel {tuple(kernel.shape)} must be [M, K] / [N, K]")
    M, K = in_feats.shape
    N = kernel.shape[0]
    acc = torch.empty(M, N, dtype=torch.int32, device=dev)
    with _Dev(dev):
        _lib.call("qvggt_i8_gemm_i32", _ptr(in_feats), _ptr(kernel), _ptr(acc), M, N, K, _stream(in_feats))
    return acc


def invoke_quant(out, input, scale):
    """Per-token int8 quantisation (``quantization.cu:81-96``); writes out and scale."""
    name = "invoke_quant"
    dev = _check_cuda(name, out, input, scale)
    _check_dtype(name, input, torch.float16)
    _contig(name, out, input, scale)
    H = input.shape[-1]
    with _Dev(dev):
        _lib.call("qvggt_invoke_quant", _ptr(out), _ptr(input), _ptr(scale), input.numel() // H, H, _stream(input))


def rms_norm_general(out, input, weight, bias, scaling, epsilon: float, use_per_token_quant: bool = True):
    """LayerNorm + int8 quantisation (``w8a8/layernorm.cu:155-191``); writes out and scaling."""
    name = "rms_norm_general"
    dev = _check_cuda(name, out, input, weight, bias, scaling)
    _check_dtype(name, input, torch.float16)
    _contig(name, out, input, weight, bias, scaling)
    H = input.shape[-1]
    with _Dev(dev):
        _lib.call("qvggt_layernorm_quant", _ptr(out), _ptr(input), _ptr(weight), _ptr(bias), _ptr(scaling),
                  input.numel() // H, H, float(epsilon), 1 if use_per_token_quant else 0, _stream(input))


def gelu_and_quant(out, input, scale_out, tmp):
    """tanh-GELU + per-token int8 (``w8a8/act.cu:77-90``); writes out, scale_out, tmp."""
    name = "gelu_and_quant"
    dev = _check_cuda(name, out, input, scale_out, tmp)
    _check_dtype(name, input, torch.float16)
    _contig(name, out, input, scale_out, tmp)
    d = input.shape[-1]
    with _Dev(dev):
        _lib.call("qvggt_gelu_quant", _ptr(out), _ptr(input), _ptr(scale_out), _ptr(tmp), input.numel() // d, d,
                  _stream(input))


def silu_and_mul(input):
    raise NotImplementedError("silu_and_mul (SwiGLU) is not part of the VGGT path")


# ---------------------------------------------------------------------- RoPE
def fused_rope_with_pos_forward_func(input, freqs, transpose_output_memory: bool):
    """Rotate-half RoPE with per-(b, s) angles (``fused_rope_with_pos.cu:122-164``).

    input [s, b, h, d] fp16 (any strides), freqs fp32 [b, s, d2].  Returns a new
    tensor [s, b, h, d]; with transpose_output_memory it is a transposed view of
    a contiguous [b, s, h, d] buffer, as in the reference.
    """
    name = "fused_rope_with_pos_forward_func"
    dev = _check_cuda(name, input, freqs)
    _check_dtype(name, input, torch.float16)
    _check_dtype(name, freqs, torch.float32)
    s, b, h, d = input.shape
    d2 = freqs.shape[-1]
    freqs = freqs.contiguous()
    if transpose_output_memory:
        out = torch.empty(b, s, h, d, dtype=input.dtype, device=dev).transpose(0, 1)
    else:
        out = torch.empty(s, b, h, d, dtype=input.dtype, device=dev)
    ist = (C.c_int64 * 4)(*input.stride())
    ost = (C.c_int64 * 4)(*out.stride())
    with _Dev(dev):
        _lib.call("qvggt_rope_with_pos", _ptr(input), _ptr(freqs), _ptr(out), s, b, h, d, d2, ist, ost,
                  _stream(input))
    return out


def rotary_embedding_neox(*args, **kw):
    raise NotImplementedError("rotary_embedding_neox (1-D LLM RoPE) is not part of the VGGT path")


def layernorm_forward_cuda(*args, **kw):
    raise NotImplementedError("layernorm_forward_cuda (T5 RMSNorm) is not part of the VGGT path")


def single_query_attention(*args, **kw):
    raise NotImplementedError("single_query_attention (decode attention) is not part of the VGGT path")


# ----------------------------------------------------------- new hot-path ops
def layernorm(x, weight, bias, eps: float = 1e-6, out=None):
    name = "layernorm"
    dev = _check_cuda(name, x, weight, bias, out)
    _check_dtype(name, x, torch.float16)
    _contig(name, x, weight, bias, out)
    H = x.shape[-1]
    _check_shape(name, weight.numel() >= H and bias.numel() >= H, f"weight / bias need {H} entries")
    if out is None:
        out = torch.empty_like(x)
    _check_shape(name, out.numel() == x.numel() and out.dtype == torch.float16, "out must match x")
    with _Dev(dev):
        _lib.call("qvggt_layernorm", _ptr(x), _ptr(weight), _ptr(bias), _ptr(out), x.numel() // H, H, float(eps),
                  _stream(x))
    return out


def qkv_rope2d(qkv, heads: int, cos_tab, sin_tab, tokens_per_frame: int = 1374, patch_start: int = 5,
               grid_w: int = 37, token_offset: int = 0, q_out=None, kv_out=None, qk_norm=None, eps: float = 1e-6):
    """Split qkv [T, 3*C] into roped q [T, C] and [k roped | v] [T, 2*C]."""
    name = "qkv_rope2d"
    dev = _check_cuda(name, qkv, cos_tab, sin_tab)
    _contig(name, qkv, cos_tab, sin_tab)
    T = qkv.numel() // qkv.shape[-1]
    Cd = qkv.shape[-1] // 3
    if q_out is None:
        q_out = torch.empty(T, Cd, dtype=torch.float16, device=dev)
    if kv_out is None:
        kv_out = torch.empty(T, 2 * Cd, dtype=torch.float16, device=dev)
    qn = qk_norm if qk_norm is not None else (None, None, None, None)
    with _Dev(dev):
        _lib.call("qvggt_qkv_rope2d", _ptr(qkv), _ptr(q_out), _ptr(kv_out), T, heads, token_offset,
                  tokens_per_frame, patch_start, grid_w, _ptr(cos_tab), _ptr(sin_tab), cos_tab.shape[0],
                  1 if qk_norm is not None else 0, _ptr(qn[0]), _ptr(qn[1]), _ptr(qn[2]), _ptr(qn[3]), float(eps),
                  _stream(qkv))
    return q_out, kv_out


IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def patchify(images, patch: int = 14, k_pad: int = 640, out=None, mean=IMAGENET_MEAN, std=IMAGENET_STD):
    """images fp16 [S, 3, H, W] -> normalised patches [S*(H/p)*(W/p), k_pad]."""
    name = "patchify"
    dev = _check_cuda(name, images)
    _contig(name, images)
    S, _, H, W = images.shape
    rows = S * (H // patch) * (W // patch)
    if out is None:
        out = torch.empty(rows, k_pad, dtype=F16_, device=dev)
    m = (C.c_float * 3)(*mean)
    s = (C.c_float * 3)(*std)
    with _Dev(dev):
        _lib.call("qvggt_patchify", _ptr(images), _ptr(out), S, H, W, patch, k_pad, m, s, _stream(images))
    return out


def assemble_tokens(src, src_rows_per_frame: int, src_row_offset: int, specials, n_special: int, two_sets: bool,
                    pos, out, S: int, P: int, frame_offset: int = 0):
    """out [S, P, C] = per-frame [specials | src rows] (+ pos)."""
    name = "assemble_tokens"
    dev = _check_cuda(name, src, specials, pos, out)
    Cd = out.shape[-1]
    with _Dev(dev):
        _lib.call("qvggt_assemble_tokens", _ptr(src), src_rows_per_frame, src_row_offset, _ptr(specials), n_special,
                  1 if two_sets else 0, _ptr(pos), _ptr(out), S, P, Cd, frame_offset, _stream(out))
    return out


F16_ = torch.float16


def attention_small(q, kv, heads: int, batches: int, L: int, out=None, k_col0: int | None = None,
                    v_col0: int | None = None):
    """Attention with head_dim 128 over L <= 256 tokens per batch (camera-head
    trunk): q [batches*L, heads*128], kv rows holding k and v (by default
    kv = [k | v]).  Returns out [batches*L, heads*128]."""
    name = "attention_small"
    dev = _check_cuda(name, q, kv, out)
    Cd = heads * 128
    if out is None:
        out = torch.empty(batches * L, Cd, dtype=torch.float16, device=dev)
    k0 = 0 if k_col0 is None else k_col0
    v0 = Cd if v_col0 is None else v_col0
    _check_rows(name, q, batches * L, Cd, "q")
    _check_rows(name, kv, batches * L, max(k0, v0) + Cd, "kv")
    _check_rows(name, out, batches * L, Cd, "out")
    with _Dev(dev):
        _lib.call("qvggt_attention_small", _ptr(q), q.stride(0), _ptr(kv), kv.stride(0), k0, v0, _ptr(out),
                  out.stride(0), batches, L, heads, _stream(q))
    return out


def attention(q, kv, heads: int, batches: int, Lq: int, Lkv: int, out=None, k_col0: int | None = None,
              v_col0: int | None = None):
    """Flash attention (head_dim 64) over token-major q [batches*Lq, heads*64]
    and kv [batches*Lkv, 2*heads*64] (= [k | v]).  Returns out [batches*Lq, heads*64]."""
    name = "attention"
    dev = _check_cuda(name, q, kv, out)
    Cd = heads * 64
    if out is None:
        out = torch.empty(batches * Lq, Cd, dtype=torch.float16, device=dev)
    k0 = 0 if k_col0 is None else k_col0
    v0 = Cd if v_col0 is None else v_col0
    _check_rows(name, q, batches * Lq, Cd, "q")
    _check_rows(name, kv, batches * Lkv, max(k0, v0) + Cd, "kv")
    _check_rows(name, out, batches * Lq, Cd, "out")
    with _Dev(dev):
        _lib.call("qvggt_attention", _ptr(q), q.stride(0), _ptr(kv), kv.stride(0), k0, v0, _ptr(out), out.stride(0),
                  batches, Lq, Lkv, heads, _stream(q))
    return out


def attention_plan(batches: int, Lq: int, keys: int, heads: int) -> tuple[int, int]:
    """(splits, scratch bytes) the library picks for this shape on the current
    device: the split count that runs the grid in the fewest waves of CTAs
    over the SMs."""
    sp = C.c_int32(0)
    nb = C.c_int64(0)
    _lib.call("qvggt_attention_plan", batches, Lq, keys, heads, C.byref(sp), C.byref(nb))
    return int(sp.value), int(nb.value)


def attention_scratch_bytes(batches: int, Lq: int, heads: int, splits: int) -> int:
    nb = C.c_int64(0)
    _lib.call("qvggt_attention_scratch_bytes", batches, Lq, heads, splits, C.byref(nb))
    return int(nb.value)


def attention_ex(q, kv, heads: int, batches: int, Lq: int, Lkv: int, out=None, k_col0: int | None = None,
                 v_col0: int | None = None, segments=None, splits: int | None = None, lse=None, lse_mode: int = 0,
                 scratch=None):
    """:func:`attention` over a subset of each batch's keys, in parts that merge exactly.

    ``segments``: up to two (start, length) key-row ranges per batch (default
    all Lkv rows).  ``splits``: CTAs per (batch, head, 256-query block), each
    over a consecutive part of the keys (None: the library's plan).  ``lse``
    (fp32 [batches, heads, Lq]): ln(sum_k exp(q.k / 8)) per row; ``lse_mode``
    1 writes it, 2 merges this call's result with an earlier call's (``out``
    and ``lse``, over other keys of the same rows) and writes both.
    ``scratch``: a uint8 CUDA tensor of at least
    :func:`attention_scratch_bytes` bytes when splits > 1 (allocated here if
    None).  Returns ``out``."""
    name = "attention_ex"
    dev = _check_cuda(name, q, kv, out, lse, scratch)
    Cd = heads * 64
    if out is None:
        out = torch.empty(batches * Lq, Cd, dtype=torch.float16, device=dev)
    k0 = 0 if k_col0 is None else k_col0
    v0 = Cd if v_col0 is None else v_col0
    _check_rows(name, q, batches * Lq, Cd, "q")
    _check_rows(name, kv, batches * Lkv, max(k0, v0) + Cd, "kv")
    _check_rows(name, out, batches * Lq, Cd, "out")
    segs = [(0, Lkv)] if segments is None else [tuple(map(int, sg)) for sg in segments if sg[1] > 0]
    _check_shape(name, 1 <= len(segs) <= 2, "one or two non-empty key segments")
    (s0, n0), (s1, n1) = segs[0], (segs[1] if len(segs) > 1 else (0, 0))
    keys = n0 + n1
    if lse_mode:
        _check_shape(name, lse is not None and lse.dtype == torch.float32 and lse.is_contiguous()
                     and lse.numel() >= batches * heads * Lq, "lse must be fp32 contiguous [batches, heads, Lq]")
    with _Dev(dev):
        if splits is None:
            splits, _ = attention_plan(batches, Lq, keys, heads)
        nbytes = attention_scratch_bytes(batches, Lq, heads, splits) if splits > 1 else 0
        if nbytes and scratch is None:
            scratch = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        if scratch is not None:
            _check_shape(name, scratch.dtype == torch.uint8 and scratch.is_contiguous() and scratch.numel() >= nbytes,
                         f"scratch must be a contiguous uint8 tensor of >= {nbytes} bytes")
        _lib.call("qvggt_attention_ex", _ptr(q), q.stride(0), _ptr(kv), kv.stride(0), k0, v0, _ptr(out),
                  out.stride(0), batches, Lq, Lkv, s0, n0, s1, n1, heads, splits, lse_mode, _ptr(lse), _ptr(scratch),
                  scratch.numel() if scratch is not None else 0, _stream(q))
    return out

