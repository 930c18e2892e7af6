"""CPU: the oracle against golden outputs of the reference's own CUDA kernels.

``tests/golden/ref_cuda_golden.npz`` was produced on a B200 by
``tests/golden/make_ref_cuda_golden.py`` running the reference kernels built
from their own sources (``oracle/build_ref.py``); inputs are regenerated here
from the same seeds.  Bounds per kernel:

* W4A16 GEMM / GEMV: the reference accumulates in fp16, the oracle in fp32:
  max-abs-rel <= 1e-2 (north-star per-linear bound).
* W8A8 GEMM epilogue: bit-exact (same fp32 operation order, int32 accumulators exact).
* rms_norm_general, invoke_quant: int8 within 1 code on <= 1e-3 of elements
  (the reference's --use_fast_math rsqrt / division), scales within 1e-3.
* gelu_and_quant: the reference is built with --use_fast_math, whose tanh is
  an approximation; near t = -1 the fp16 `1 + t` cancellation turns its 1-ulp
  differences into larger ones: tmp within 1e-3 absolute, int8 within 1 code.
* fused_rope_with_pos: the reference's fast-math sincos: within 2e-3 absolute.
"""
import os

import numpy as np
import pytest
import torch

from oracle import awq, rope as orope, w8a8 as ow

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(HERE, "golden", "ref_cuda_golden.npz"))


@pytest.fixture(scope="module")
def cases():
    from tests.golden.make_ref_cuda_golden import cases as c
    return c()


@pytest.mark.parametrize("name", ["gemm_a", "gemm_b"])
def test_gemm(gold, cases, name):
    d = cases[name]
    ref = awq.w4a16_linear(d["x"], d["qweight"], d["scales"], d["scaled_zeros"], 128)
    assert awq.max_abs_rel(torch.from_numpy(gold[f"{name}_y"].astype(np.float32)), ref) <= 1e-2


@pytest.mark.parametrize("m", [1, 7])
def test_gemv(gold, cases, m):
    d = cases["gemm_a"]
    ref = awq.w4a16_linear(d["x"][:m], d["qweight"], d["scales"], d["scaled_zeros"], 128)
    assert awq.max_abs_rel(torch.from_numpy(gold[f"gemv_m{m}_y"].astype(np.float32)), ref) <= 1e-2


@pytest.mark.parametrize("bias", [False, True])
def test_w8a8_bit_exact(gold, cases, bias):
    d = cases["w8a8"]
    y = ow.w8a8_gemm(d["a"], d["w"], d["ws"], d["as_"], d["bias"] if bias else None)
    g = gold["w8a8_bias_y" if bias else "w8a8_y"]
    assert np.array_equal(y.view(np.uint16), g.view(np.uint16))


def _close_i8(q, g, frac=1e-3):
    d = np.abs(q.astype(np.int32) - g.astype(np.int32))
    assert d.max() <= 1
    assert (d > 0).mean() <= frac


def test_invoke_quant(gold, cases):
    q, s = ow.invoke_quant(cases["quant"]["x"])
    _close_i8(q, gold["quant_q"])
    assert np.array_equal(s, gold["quant_s"])


def test_rms_norm_general(gold, cases):
    d = cases["ln"]
    q, s = ow.rms_norm_general(d["x"], d["w"], d["b"], 1e-6)
    _close_i8(q, gold["ln_q"])
    assert np.abs(s.astype(np.float32) - gold["ln_s"].astype(np.float32)).max() <= 1e-3 * np.abs(s).max()


def test_rms_norm_general_per_tensor(gold, cases):
    d = cases["ln"]
    xf = torch.from_numpy(d["x"]).float()
    mu = xf.mean(-1, keepdim=True)
    var = (xf * xf).mean(-1, keepdim=True) - mu * mu
    ln = ((xf - mu) * torch.rsqrt(var + 1e-6) * torch.from_numpy(d["w"]).float()).half().float()
    _close_i8(ow.cvt_rni_sat_s8((ln * 20.0).numpy()), gold["ln_tensor_q"], frac=2e-3)


def test_gelu_and_quant(gold, cases):
    q, s, t = ow.gelu_and_quant(cases["gelu"]["x"])
    g = gold["gelu_tmp"].astype(np.float32)
    assert np.all(np.abs(t.astype(np.float32) - g) <= 1e-3 + 1e-3 * np.abs(g))
    assert (t.view(np.uint16) != gold["gelu_tmp"].view(np.uint16)).mean() <= 5e-3
    _close_i8(q, gold["gelu_q"])
    assert np.abs(s.astype(np.float32) - gold["gelu_s"].astype(np.float32)).max() <= 1e-3 * np.abs(s).max()


@pytest.mark.parametrize("tr", [0, 1])
def test_fused_rope(gold, cases, tr):
    d = cases["rope"]
    y = orope.fused_rope_with_pos(torch.from_numpy(d["x"]), torch.from_numpy(d["freqs"]), bool(tr)).numpy()
    assert np.abs(y.astype(np.float32) - gold[f"rope_y_{tr}"].astype(np.float32)).max() <= 2e-3


def test_oracle_dequant_equals_reference_kernel_bit_for_bit():
    """The reference's ``gemm_forward_cuda_new`` with A = I returns its
    dequantised weight matrix; the oracle's restatement of the unpack and the
    fp16 fma (``oracle.awq.dequantize``) must equal it bit for bit."""
    import os
    import numpy as np
    from oracle import awq
    from tests.golden.make_ref_cuda_golden import gemm_pin_cases
    gold = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_cuda_gemm_pins.npz"))
    d = gemm_pin_cases()["eye"]
    deq = awq.dequantize(d["qweight"], d["scales"], d["scaled_zeros"], 128)      # [N, K] fp16
    assert np.array_equal(np.ascontiguousarray(deq.T).view(np.uint16), gold["eye_y"].view(np.uint16))


BF16_PINS = os.path.join(HERE, "golden", "ref_cuda_bf16_pins.npz")


@pytest.mark.skipif(not os.path.exists(BF16_PINS), reason="bf16 reference pins not generated")
def test_oracle_bf16_dequant_equals_reference_kernel_bit_for_bit():
    """The reference's bf16 ``gemm_forward_cuda_new`` with A = I returns its
    bf16 dequantised weights; ``oracle.awq.dequantize_bf16`` (the bf16 unpack
    and one bf16x2 fma, ``dequantize.cuh:53-90``) must equal them bit for bit."""
    from tests.golden.make_ref_cuda_golden import bf16_pin_cases
    d = bf16_pin_cases()["eye"]
    deq = awq.dequantize_bf16(d["qweight"], d["scales"], d["scaled_zeros"], 128)      # [N, K]
    assert np.array_equal(awq.bf16_bits(np.ascontiguousarray(deq.T)), np.load(BF16_PINS)["eye_y"])


@pytest.mark.skipif(not os.path.exists(BF16_PINS), reason="bf16 reference pins not generated")
def test_oracle_bf16_linear_near_reference_kernels():
    """The float64 oracle against the reference's bf16 GEMM (fp32 accumulation:
    max-abs-rel <= 8e-3) and GEMV (bf16 accumulation: rel-L2 <= 2e-2)."""
    from tests.golden.make_ref_cuda_golden import bf16_pin_cases
    d = bf16_pin_cases()["lin"]
    pins = np.load(BF16_PINS)
    ref = awq.w4a16_linear_bf16(d["x"], d["qweight"], d["scales"], d["scaled_zeros"], 128)
    y = awq.from_bf16_bits(pins["gemm_y"])
    assert awq.max_abs_rel(torch.from_numpy(y), torch.from_numpy(ref)) <= 8e-3
    for m in (1, 5):
        y = awq.from_bf16_bits(pins[f"gemv_m{m}_y"])
        assert awq.rel_l2(torch.from_numpy(y), torch.from_numpy(ref[:m])) <= 2e-2


def test_oracle_bf16_round_matches_torch():
    """oracle.awq.bf16_round (one rounding from float64) equals torch's
    float32 -> bf16 conversion on float32 inputs, ties included."""
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(20000) * 10.0 ** rng.integers(-6, 6, 20000)).astype(np.float32)
    x[:4] = [1 + 2 ** -8, 1 + 3 * 2 ** -8, -(1 + 2 ** -8), 0.0]
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(awq.bf16_round(x.astype(np.float64)), want)
