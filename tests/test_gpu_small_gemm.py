"""GPU parity of the small-M split-K GEMM (qvggt_small_linear) against the CPU oracle.

Shapes are those of the camera-head trunk (dim 2048: qkv 2048->6144, proj
2048->2048, fc1 2048->8192, fc2 8192->2048) with one row per frame, plus edge
row counts for every padded tile height (16, 32, 64, 128, 256).
Tolerances: max-abs-rel <= 2e-3 against the fp32-accumulated oracle (the
per-linear bound is 1e-2); the split-K sum order is fixed, so repeated calls
are bit-identical.
"""
import numpy as np
import pytest
import torch

from oracle import awq, model as om

pytestmark = pytest.mark.gpu

DEV = "cuda"
_CACHE = {}


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from qvggt_b200 import _lib as L
    L.load()
    yield


def _lin(N, K, G=128, seed=0):
    key = (N, K, G, seed)
    if key not in _CACHE:
        lin = awq.make_quantized_linear(N, K, G, seed=seed)
        t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(DEV) for k, v in lin.items()
             if k in ("qweight", "scales", "scaled_zeros", "bias")}
        deq = torch.from_numpy(awq.dequantize(lin["qweight"], lin["scales"], lin["scaled_zeros"], G).astype(np.float32))
        _CACHE[key] = (lin, t, deq)
    return _CACHE[key]


def _ref(x, deq, bias=None):
    y = om.r16(x.float() @ deq.T)
    if bias is not None:
        y = om.r16(y.float() + torch.from_numpy(np.asarray(bias)).float())
    return y


@pytest.mark.parametrize("M", [1, 17, 32, 64, 100, 200, 256])
@pytest.mark.parametrize("N,K", [(6144, 2048), (2048, 2048), (2048, 8192)])
def test_small_w4_matches_oracle(M, N, K):
    from qvggt_b200 import awq_inference_engine as eng
    lin, t, deq = _lin(N, K, seed=N + K)
    x = torch.randn(M, K, dtype=torch.float16)
    y = eng.small_linear(x.to(DEV), t["qweight"], t["scales"], t["scaled_zeros"], t["bias"]).cpu()
    assert awq.max_abs_rel(y, _ref(x, deq, lin["bias"])) <= 2e-3


@pytest.mark.parametrize("M", [20, 64, 256])
def test_small_f16_matches_oracle(M):
    from qvggt_b200 import awq_inference_engine as eng
    N, K = 2048, 1024
    w = (torch.randn(N, K) * 0.02).half()
    b = (torch.randn(N) * 0.01).half()
    x = torch.randn(M, K, dtype=torch.float16)
    y = eng.small_linear(x.to(DEV), w.to(DEV), bias=b.to(DEV)).cpu()
    ref = om.QLinear("f16", weight=w, bias=b)(x)
    assert awq.max_abs_rel(y, ref) <= 2e-3


@pytest.mark.parametrize("kind", ["w4", "f16"])
def test_small_epilogues_gelu_and_residual(kind):
    from qvggt_b200 import awq_inference_engine as eng
    M, N, K = 40, 2048, 2048
    lin, t, deq = _lin(N, K, seed=3)
    x = torch.randn(M, K, dtype=torch.float16)
    if kind == "w4":
        args = (t["qweight"], t["scales"], t["scaled_zeros"])
        w_ref = deq
    else:
        w16 = deq.half()
        args = (w16.to(DEV),)
        w_ref = w16.float()
    y_lin = _ref(x, w_ref, lin["bias"])
    y = eng.small_linear(x.to(DEV), *args, bias=t["bias"], act="gelu").cpu()
    assert awq.max_abs_rel(y, om.gelu_erf(y_lin)) <= 2e-3
    resid = torch.randn(M, N, dtype=torch.float16)
    gamma = torch.full((N,), 0.37, dtype=torch.float16)
    r_dev = resid.to(DEV)
    eng.small_linear(x.to(DEV), *args, bias=t["bias"], residual=r_dev, gamma=gamma.to(DEV))
    ref2 = om.r16(resid.float() + om.r16(y_lin.float() * gamma.float()).float())
    assert awq.max_abs_rel(r_dev.cpu(), ref2) <= 2e-3


def test_small_repeatable_and_equal_to_large_kernel():
    """Two calls are bit-identical (partials are summed in cluster-rank order);
    the large tcgen05 kernel on the same rows agrees within the per-linear
    tolerance."""
    from qvggt_b200 import _lib as L
    M, N, K = 48, 6144, 2048
    lin, t, deq = _lin(N, K, seed=11)
    x = torch.randn(M, K, dtype=torch.float16, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    outs = []
    for _ in range(2):
        y = torch.empty(M, N, dtype=torch.float16, device=DEV)
        L.call("qvggt_small_linear", 0, x.data_ptr(), K, t["qweight"].data_ptr(), t["scales"].data_ptr(),
               t["scaled_zeros"].data_ptr(), t["scales"].shape[0], 128, t["bias"].data_ptr(), y.data_ptr(), N, M, N,
               K, 0, None, 0, None, st)
        outs.append(y.cpu())
    assert torch.equal(outs[0], outs[1])
    big = torch.empty(M, N, dtype=torch.float16, device=DEV)
    L.call("qvggt_w4a16_linear_ex", x.data_ptr(), K, t["qweight"].data_ptr(), t["scales"].data_ptr(),
           t["scaled_zeros"].data_ptr(), t["bias"].data_ptr(), big.data_ptr(), N, M, N, K, t["scales"].shape[0], 128,
           0, None, 0, None, st)
    assert awq.max_abs_rel(outs[0], big.cpu()) <= 2e-3
    assert awq.max_abs_rel(outs[0], _ref(x.cpu(), deq, lin["bias"])) <= 2e-3


def test_small_argument_checks():
    from qvggt_b200 import _lib as L
    M, N, K = 32, 2048, 2048
    lin, t, _ = _lin(N, K, seed=5)
    x = torch.randn(300, K, dtype=torch.float16, device=DEV)
    y = torch.empty(300, N, dtype=torch.float16, device=DEV)
    st = torch.cuda.current_stream().cuda_stream

    def call(M=M, N=N, K=K, ldo=N, act=0, resid=None):
        L.call("qvggt_small_linear", 0, x.data_ptr(), K, t["qweight"].data_ptr(), t["scales"].data_ptr(),
               t["scaled_zeros"].data_ptr(), t["scales"].shape[0], 128, None, y.data_ptr(), ldo, M, N, K, act,
               resid, N if resid else 0, None, st)

    with pytest.raises(L.QvggtError, match="M=300"):
        call(M=300)
    with pytest.raises(L.QvggtError, match="multiple of 128"):
        call(N=2000)
    with pytest.raises(L.QvggtError, match="multiple of 64"):
        call(K=2000)
    with pytest.raises(L.QvggtError, match="in place"):
        call(resid=x.data_ptr())
    call()
    torch.cuda.synchronize()
