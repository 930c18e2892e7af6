"""Oracle: W8A8 per-token int8 quantisation chain (CPU).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Reference: DDsacu/QVGGT ``qvggt/runtime/awq_inference_engine/csrc/w8a8/``.
fp16 ("half") operations of the reference are emulated one at a time: the
exact result is formed in float64 and rounded once to fp16, which is what a
correctly rounded ``__hmul`` / ``__hadd`` / ``__hfma`` produces.
"""
from __future__ import annotations

import math

import numpy as np
import torch

F16 = np.float16


def cvt_rni_sat_s8(x) -> np.ndarray:
    """``cvt.rni.sat.s8.f32`` (``w8a8/utils.cuh:75-80``): round half to even,
    saturate to [-128, 127]; NaN -> 0."""
    x = np.asarray(x, dtype=np.float64)
    r = np.rint(x)
    r = np.where(np.isnan(r), 0.0, r)
    return np.clip(r, -128, 127).astype(np.int8)


def h(x) -> np.ndarray:
    """Round to fp16 (one rounding from float64)."""
    return np.asarray(x, dtype=np.float64).astype(F16)


def hmul(a, b):
    return h(np.asarray(a, np.float64) * np.asarray(b, np.float64))


def hadd(a, b):
    return h(np.asarray(a, np.float64) + np.asarray(b, np.float64))


def invoke_quant(x):
    """Per-token dynamic int8 quantisation (``w8a8/quantization.cu:41-78``).

    amax = max|x| (fp32, start 0); scale = half(amax / 127);
    q = rni_sat(x * (127 / amax)) in fp32.
    Returns (q int8 [T, H], scale fp16 [T]).
    """
    x32 = np.asarray(x, dtype=F16).astype(np.float32)
    T, H = x32.reshape(-1, x32.shape[-1]).shape
    x32 = x32.reshape(T, H)
    amax = np.abs(x32).max(axis=1).astype(np.float32)
    scale = (amax / np.float32(127.0)).astype(np.float32).astype(F16)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = (np.float32(127.0) / amax).astype(np.float32)
        q = cvt_rni_sat_s8((x32 * inv[:, None]).astype(np.float32))
    return q, scale


def rms_norm_general(x, gamma, beta, eps: float):
    """LayerNorm + per-token int8 (``w8a8/layernorm.cu:20-191``, per-token path).

    mean = E[x], var = E[x^2] - mean^2 (fp32), rs = 1/sqrt(var + eps);
    ln = (x - mean) * rs * gamma + beta (fp32);
    amax over the fp16-rounded ln values, starting from half(1e-6) (``:100-113``);
    q = rni_sat(ln_fp32 * (127 / amax)) (``:130-145``, ln recomputed in fp32);
    scale = half(amax / 127) (``:146-149``).
    Returns (q int8 [T, H], scale fp16 [T]).
    """
    x32 = np.asarray(x, dtype=F16).astype(np.float32)
    H = x32.shape[-1]
    x32 = x32.reshape(-1, H)
    g = np.asarray(gamma, dtype=F16).astype(np.float32)
    b = np.zeros(H, np.float32) if beta is None else np.asarray(beta, dtype=F16).astype(np.float32)
    mean = (x32.astype(np.float64).sum(axis=1) / H).astype(np.float32)
    msq = ((x32.astype(np.float64) ** 2).sum(axis=1) / H).astype(np.float32)
    var = (msq - mean * mean).astype(np.float32)
    rs = (1.0 / np.sqrt(var.astype(np.float64) + eps)).astype(np.float32)
    ln = ((x32 - mean[:, None]) * rs[:, None] * g[None, :] + b[None, :]).astype(np.float32)
    amax0 = np.float32(F16(1e-6))
    amax = np.maximum(np.abs(ln.astype(F16)).astype(np.float32).max(axis=1), amax0)
    inv = (np.float32(127.0) / amax).astype(np.float32)
    q = cvt_rni_sat_s8((ln * inv[:, None]).astype(np.float32))
    scale = (amax / np.float32(127.0)).astype(np.float32).astype(F16)
    return q, scale


def gelu_fast_h(x):
    """fp16 tanh-GELU ``gelu_fast<half>`` (``w8a8/act.cu:22-28``), op by op in fp16.

    ``(T)1.0 + (T)(0.044715 * f) * x`` is a half multiply followed by a half
    add, which nvcc contracts (default -fmad=true) into one fp16 fma: one
    rounding of b*x + 1.
    """
    x = np.asarray(x, dtype=F16)
    f = x
    a = hmul(F16(0.79788456), f)
    b = hmul(F16(0.044715), f)
    d = h(b.astype(np.float64) * x.astype(np.float64) + 1.0)
    e = hmul(a, d)
    t = h(np.tanh(e.astype(np.float64)))
    half_x = hmul(F16(0.5), x)
    return hmul(half_x, hadd(F16(1.0), t))


def gelu_and_quant(x):
    """Fused tanh-GELU + per-token int8 (``w8a8/act.cu:30-74``, per-token path).

    tmp = gelu_fast(x) (fp16); amax over ``t > 0.0001 ? t : -t`` (the reference's
    ``zero = 0.0001`` quirk, ``:42,49``; fp32 compare, start 0);
    scale = half(amax / 127); q = rni_sat(float(half(127/amax) * tmp)) with an
    fp16 multiply (``:62-66``).  Returns (q int8, scale fp16 [T], tmp fp16).
    """
    x = np.asarray(x, dtype=F16)
    H = x.shape[-1]
    x = x.reshape(-1, H)
    t = gelu_fast_h(x)
    zero = F16(0.0001)
    a = np.where(t > zero, t, -t).astype(np.float32)
    amax = np.maximum(a.max(axis=1), np.float32(0.0))
    scale = (amax / np.float32(127.0)).astype(np.float32).astype(F16)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = h((np.float32(127.0) / amax).astype(np.float32))
    prod = hmul(inv[:, None], t)
    q = cvt_rni_sat_s8(prod.astype(np.float32))
    return q, scale, t


def int8_gemm_i32(a_i8, w_i8) -> np.ndarray:
    """Exact int32 accumulators acc[m, n] = sum_k a[m,k] * w[n,k]."""
    a = torch.from_numpy(np.asarray(a_i8, dtype=np.int8).astype(np.int64))
    w = torch.from_numpy(np.asarray(w_i8, dtype=np.int8).astype(np.int64))
    acc = a @ w.t()
    return acc.numpy().astype(np.int32)


def w8a8_epilogue(acc_i32, wscale, ascale, bias=None) -> np.ndarray:
    """Rescale epilogue of ``dense_kernel0[_fuse_bias]``.

    no bias (``w8a8_gemm_cuda.cu:868-873``): y = float(acc) * (ws * as);
    bias    (``w8a8_gemm_cuda.cu:551-556``): y = (float(acc) * ws) * as + bias
    (the multiply-add contracts to one fma under -O3), all fp32, then fp16 RN.
    """
    acc = np.asarray(acc_i32, dtype=np.int32).astype(np.float32)
    ws = np.asarray(wscale, dtype=F16).astype(np.float32)[None, :]
    as_ = np.asarray(ascale, dtype=F16).astype(np.float32)[:, None]
    if bias is None:
        y = acc * (ws * as_).astype(np.float32)
        return y.astype(np.float32).astype(F16)
    b = np.asarray(bias, dtype=F16).astype(np.float32)[None, :]
    prod = (acc * ws).astype(np.float32)
    y = (prod.astype(np.float64) * as_.astype(np.float64) + b.astype(np.float64)).astype(np.float32)
    return y.astype(F16)


def w8a8_gemm(a_i8, w_i8, wscale, ascale, bias=None) -> np.ndarray:
    return w8a8_epilogue(int8_gemm_i32(a_i8, w_i8), wscale, ascale, bias)


def quantize_weight_per_channel(w) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric per-output-channel int8: scale = max|W|/127."""
    w = np.asarray(w, dtype=np.float32)
    s = (np.abs(w).max(axis=1) / 127.0).astype(np.float32)
    s16 = s.astype(F16)
    q = cvt_rni_sat_s8(w / np.maximum(s16.astype(np.float32), 1e-12)[:, None])
    return q, s16


def gelu_erf_f32(x):
    x = np.asarray(x, dtype=np.float64)
    return 0.5 * x * (1.0 + np.vectorize(math.erf)(x / math.sqrt(2.0)))
