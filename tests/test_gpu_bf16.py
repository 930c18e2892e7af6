"""GPU parity of the bf16 W4A16 path: the reference's bf16 instantiation of
gemm_forward_cuda_new / gemv_forward_cuda_new (``dispatch_utils.cuh:7-17``)
against the CPU oracle and the reference kernels' own outputs.

Tolerances: bit-exact for the bf16 dequantisation (identity activations make
every output one dequantised weight, in every kernel: the three large-M
configurations, the small-M split-K kernel and the GEMV); for random
activations max-abs-rel <= 8e-3 against the float64 oracle (fp32
accumulation plus one bf16 rounding, 2^-8 relative at most per element) and
rel-L2 <= 2e-2 against the reference kernels' outputs (its GEMV sums in bf16).
"""
import os

import numpy as np
import pytest
import torch

from oracle import awq

pytestmark = pytest.mark.gpu

DEV = "cuda"
PINS = os.path.join(os.path.dirname(__file__), "golden", "ref_cuda_bf16_pins.npz")


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from qvggt_b200 import _lib as L
    L.load()
    yield


def _bf(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).to(DEV)


def _weights(d):
    return (torch.from_numpy(np.ascontiguousarray(d["qweight"])).to(DEV), _bf(d["scales"]), _bf(d["scaled_zeros"]))


def _bits(y):
    return awq.bf16_bits(y.float().cpu().numpy())


def _cases():
    from tests.golden.make_ref_cuda_golden import bf16_pin_cases
    return bf16_pin_cases()


def test_bf16_dequant_bit_exact_every_kernel():
    """A = identity rows: every GEMM configuration, the small-M kernel and the
    GEMV return deq_bf16(W)^T bit for bit, equal to the oracle and to the
    reference kernel's own output."""
    from qvggt_b200 import _lib
    from qvggt_b200 import awq_inference_engine as eng
    d = _cases()["eye"]
    qw, s, z = _weights(d)
    want = awq.bf16_bits(awq.dequantize_bf16(d["qweight"], d["scales"], d["scaled_zeros"], 128).T)  # [K, N]
    if os.path.exists(PINS):
        assert np.array_equal(want, np.load(PINS)["eye_y"])
    eye = _bf(d["x"])
    try:
        for cfg in (1, 2, 3):   # CTA pairs, 1-SM 256-wide, 1-SM 128-wide
            _lib.call("qvggt_set_gemm_config", cfg)
            y = eng.gemm_forward_cuda_new(eye, qw, s, z)
            assert y.dtype == torch.bfloat16
            assert np.array_equal(_bits(y), want), cfg
    finally:
        _lib.call("qvggt_set_gemm_config", 0)
    for rows in (16, 100, 256):     # the split-K small-M kernel
        y = eng.gemm_forward_cuda_new(eye[:rows].contiguous(), qw, s, z)
        assert np.array_equal(_bits(y), want[:rows]), rows
    for m in (1, 3, 7, 16):        # the GEMV
        K, N = eye.shape[1], qw.shape[0] * 4
        y = eng.gemv_forward_cuda_new(eye[:m].contiguous(), qw, s, z, m, N, K, 128)
        assert np.array_equal(_bits(y), want[:m]), m


@pytest.mark.parametrize("M", [1, 5, 64, 200, 300, 1024])
def test_bf16_linear_matches_oracle(M):
    from qvggt_b200 import awq_inference_engine as eng
    N, K = 512, 1024
    lin = awq.make_quantized_linear_bf16(N, K, 128, seed=40 + M, bias=True)
    x = awq.bf16_round(np.random.default_rng(M).standard_normal((M, K)))
    qw, s, z = _weights(lin)
    ref = awq.w4a16_linear_bf16(x, lin["qweight"], lin["scales"], lin["scaled_zeros"], 128)
    if M <= 16:
        y = eng.gemv_forward_cuda_new(_bf(x), qw, s, z, M, N, K, 128)
    else:
        y = eng.gemm_forward_cuda_new(_bf(x), qw, s, z)
    assert awq.max_abs_rel(y.float().cpu(), torch.from_numpy(ref)) <= 8e-3
    # with the bias: bf16(bf16(acc) + bias), through the routed linear
    yb = eng.w4a16_linear(_bf(x), qw, s, z, bias=_bf(lin["bias"]))
    refb = awq.w4a16_linear_bf16(x, lin["qweight"], lin["scales"], lin["scaled_zeros"], 128, bias=lin["bias"])
    assert yb.dtype == torch.bfloat16
    assert awq.max_abs_rel(yb.float().cpu(), torch.from_numpy(refb)) <= 8e-3


@pytest.mark.skipif(not os.path.exists(PINS), reason="bf16 reference pins not generated")
def test_bf16_matches_reference_kernels():
    """Against the reference's own bf16 GEMM (M = 300, gemm_w4a16_T2) and GEMV
    (m = 1, 5) outputs on the same inputs."""
    from qvggt_b200 import awq_inference_engine as eng
    d = _cases()["lin"]
    pins = np.load(PINS)
    qw, s, z = _weights(d)
    x = _bf(d["x"])
    y = eng.gemm_forward_cuda_new(x, qw, s, z)
    ref = torch.from_numpy(awq.from_bf16_bits(pins["gemm_y"]))
    assert awq.rel_l2(y.float().cpu(), ref) <= 2e-2
    K, N = x.shape[1], qw.shape[0] * 4
    for m in (1, 5):
        y = eng.gemv_forward_cuda_new(x[:m].contiguous(), qw, s, z, m, N, K, 128)
        ref = torch.from_numpy(awq.from_bf16_bits(pins[f"gemv_m{m}_y"]))
        assert awq.rel_l2(y.float().cpu(), ref) <= 2e-2


def test_bf16_rejections():
    """Mixed dtypes raise (the reference's TORCH_CHECKs); fused activation /
    residual epilogues are fp16 only."""
    from qvggt_b200 import awq_inference_engine as eng
    lin = awq.make_quantized_linear_bf16(256, 256, 128, seed=1, bias=False)
    qw, s, z = _weights(lin)
    x = torch.randn(8, 256, device=DEV).to(torch.bfloat16)
    with pytest.raises(TypeError):
        eng.gemm_forward_cuda_new(x, qw, s.half(), z.half())
    with pytest.raises(TypeError):
        eng.gemv_forward_cuda_new(x[:2], qw, s, z.half(), 2, 256, 256, 128)
    with pytest.raises(NotImplementedError):
        eng.w4a16_linear(x, qw, s, z, act="gelu")
