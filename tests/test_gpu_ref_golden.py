"""GPU: this repository's kernels against golden outputs of the reference's own
CUDA kernels (run on a B200, ``tests/golden/make_ref_cuda_golden.py``), on the
same seeded inputs.  Bounds as in ``test_oracle_ref_golden.py``; the W8A8
epilogue must be bit-exact."""
import os

import numpy as np
import pytest
import torch

from oracle import awq

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
DEV = "cuda"


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(HERE, "golden", "ref_cuda_golden.npz"))


@pytest.fixture(scope="module")
def cases():
    from tests.golden.make_ref_cuda_golden import cases as c
    return c()


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("name", ["gemm_a", "gemm_b"])
def test_gemm_vs_reference_kernel(gold, cases, name):
    from qvggt_b200 import awq_inference_engine as eng
    d = cases[name]
    y = eng.gemm_forward_cuda_new(t(d["x"]), t(d["qweight"]), t(d["scales"]), t(d["scaled_zeros"])).cpu()
    # reference accumulates in fp16: compare both against each other within the per-linear bound
    assert awq.max_abs_rel(y, torch.from_numpy(gold[f"{name}_y"].astype(np.float32))) <= 1e-2


@pytest.mark.parametrize("m", [1, 7])
def test_gemv_vs_reference_kernel(gold, cases, m):
    from qvggt_b200 import awq_inference_engine as eng
    d = cases["gemm_a"]
    K, N = d["x"].shape[1], d["qweight"].shape[0] * 4
    y = eng.gemv_forward_cuda_new(t(d["x"][:m]), t(d["qweight"]), t(d["scales"]), t(d["scaled_zeros"]), m, N, K,
                                  128).cpu()
    assert awq.max_abs_rel(y, torch.from_numpy(gold[f"gemv_m{m}_y"].astype(np.float32))) <= 1e-2


@pytest.mark.parametrize("bias", [False, True])
def test_w8a8_vs_reference_kernel_bit_exact(gold, cases, bias):
    from qvggt_b200 import awq_inference_engine as eng
    d = cases["w8a8"]
    out = torch.empty(200, 256, dtype=torch.float16, device=DEV)
    if bias:
        eng.w8a8_gemm_fuse_bias_forward_cuda(t(d["a"]), t(d["w"]), t(d["ws"]), t(d["as_"]), out, t(d["bias"]))
    else:
        eng.w8a8_gemm_forward_cuda(t(d["a"]), t(d["w"]), t(d["ws"]), t(d["as_"]), out)
    g = gold["w8a8_bias_y" if bias else "w8a8_y"]
    assert np.array_equal(out.cpu().numpy().view(np.uint16), g.view(np.uint16))


def _close_i8(q, g, frac=1e-3):
    d = np.abs(q.astype(np.int32) - g.astype(np.int32))
    assert d.max() <= 1
    assert (d > 0).mean() <= frac


def test_quant_chain_vs_reference_kernels(gold, cases):
    from qvggt_b200 import awq_inference_engine as eng
    x = t(cases["quant"]["x"])
    q = torch.empty(x.shape, dtype=torch.int8, device=DEV)
    s = torch.empty(x.shape[0], dtype=torch.float16, device=DEV)
    eng.invoke_quant(q, x, s)
    _close_i8(q.cpu().numpy(), gold["quant_q"])
    assert np.array_equal(s.cpu().numpy(), gold["quant_s"])
    d = cases["ln"]
    x = t(d["x"])
    q = torch.empty(x.shape, dtype=torch.int8, device=DEV)
    s = torch.empty(x.shape[0], dtype=torch.float16, device=DEV)
    eng.rms_norm_general(q, x, t(d["w"]), t(d["b"]), s, 1e-6, True)
    _close_i8(q.cpu().numpy(), gold["ln_q"])
    assert np.abs(s.cpu().numpy().astype(np.float32) - gold["ln_s"].astype(np.float32)).max() <= 1e-3 * np.abs(
        gold["ln_s"].astype(np.float32)).max()
    q2 = torch.empty(x.shape, dtype=torch.int8, device=DEV)
    s2 = torch.tensor([20.0], dtype=torch.float16, device=DEV)
    eng.rms_norm_general(q2, x, t(d["w"]), t(d["b"]), s2, 1e-6, False)
    _close_i8(q2.cpu().numpy(), gold["ln_tensor_q"], frac=2e-3)
    x = t(cases["gelu"]["x"])
    q = torch.empty(x.shape, dtype=torch.int8, device=DEV)
    s = torch.empty(x.shape[0], dtype=torch.float16, device=DEV)
    tmp = torch.empty(x.shape, dtype=torch.float16, device=DEV)
    eng.gelu_and_quant(q, x, s, tmp)
    g = gold["gelu_tmp"].astype(np.float32)
    assert np.all(np.abs(tmp.cpu().numpy().astype(np.float32) - g) <= 1e-3 + 1e-3 * np.abs(g))
    _close_i8(q.cpu().numpy(), gold["gelu_q"])


@pytest.mark.parametrize("tr", [False, True])
def test_rope_vs_reference_kernel(gold, cases, tr):
    from qvggt_b200 import awq_inference_engine as eng
    d = cases["rope"]
    y = eng.fused_rope_with_pos_forward_func(t(d["x"]), t(d["freqs"]), tr).cpu().contiguous().numpy()
    assert np.abs(y.astype(np.float32) - gold[f"rope_y_{int(tr)}"].astype(np.float32)).max() <= 2e-3


# ------------------------------------------------ GEMM pins (reference kernel)
PINS = os.path.join(HERE, "golden", "ref_cuda_gemm_pins.npz")


@pytest.fixture(scope="module")
def pins():
    from tests.golden.make_ref_cuda_golden import gemm_pin_cases
    return np.load(PINS), gemm_pin_cases()


def test_gemm_identity_bit_exact_vs_reference_kernel(pins):
    """A = I: both kernels return the dequantised weight matrix; ours (fp32
    accumulation) and the reference's (fp16) are exact here, so every int4
    unpack and fp16 fma dequantisation must agree bit for bit."""
    from qvggt_b200 import awq_inference_engine as eng
    gold, c = pins
    d = c["eye"]
    y = eng.gemm_forward_cuda_new(t(d["x"]), t(d["qweight"]), t(d["scales"]), t(d["scaled_zeros"])).cpu().numpy()
    assert np.array_equal(y.view(np.uint16), gold["eye_y"].view(np.uint16))


def test_gemm_config0_vs_reference_kernel(pins):
    """BASELINE config 0 (1374 x 1024 -> 4096): within the per-linear bound of
    the reference's fp16-accumulating kernel on the fixture's rows."""
    from qvggt_b200 import awq_inference_engine as eng
    from tests.golden.make_ref_cuda_golden import C0_ROWS
    gold, c = pins
    d = c["c0"]
    y = eng.gemm_forward_cuda_new(t(d["x"]), t(d["qweight"]), t(d["scales"]), t(d["scaled_zeros"]))
    got = y[torch.tensor(C0_ROWS, device=DEV)].cpu()
    assert awq.max_abs_rel(got, torch.from_numpy(gold["c0_rows_y"].astype(np.float32))) <= 1e-2
