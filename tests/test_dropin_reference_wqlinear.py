"""CPU: the reference's OWN ``WQLinear`` runs on this shim unchanged.

The reference's ``qvggt/runtime/awq/qmodule.py`` is imported from the reference
checkout with ``sys.modules["awq_inference_engine"]`` set to
``qvggt_b200.awq_inference_engine`` (the one-line switch a QVGGT maintainer
makes to use this library).
Without a GPU, the shim's CUDA-only guards are relaxed and the C-ABI call is
recorded instead of made; the test then checks that ``WQLinear.forward``
(``qmodule.py:333-369``) reaches ``gemv_forward_cuda_new`` for fewer than 8
rows and ``gemm_forward_cuda_new`` otherwise, and that the library entry point
receives each of the reference's arguments in the right place.

Skipped when the reference checkout is absent (``oracle.refpath``).
"""
import ctypes
import importlib.util
import sys

import pytest
import torch

from oracle.refpath import reference_path
from qvggt_b200 import _lib
from qvggt_b200 import awq_inference_engine as eng

REF = reference_path()
pytestmark = pytest.mark.skipif(REF is None, reason="reference checkout not present")


class _NoDev:
    def __init__(self, dev):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


@pytest.fixture
def ref_qmodule(monkeypatch):
    import os
    calls = []
    monkeypatch.setitem(sys.modules, "awq_inference_engine", eng)
    monkeypatch.setattr(eng, "_check_cuda", lambda name, *ts: torch.device("cpu"))
    monkeypatch.setattr(eng, "_Dev", _NoDev)
    monkeypatch.setattr(eng, "_stream", lambda t: ctypes.c_void_p(0))
    monkeypatch.setattr(_lib, "call", lambda name, *args: calls.append((name, args)))
    path = os.path.join(REF, "qvggt", "runtime", "awq", "qmodule.py")
    spec = importlib.util.spec_from_file_location("_reference_qmodule", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod, calls


def _ptr(a):
    return a.value if isinstance(a, ctypes.c_void_p) else a


def _ref_linear(mod, K=1024, N=512, G=128):
    lin = mod.WQLinear(4, G, K, N, True, "cpu")
    g = torch.Generator().manual_seed(0)
    lin.qweight = torch.randint(-32768, 32767, lin.qweight.shape, generator=g, dtype=torch.int32).to(torch.int16)
    lin.scales = torch.rand(lin.scales.shape, generator=g).half()
    lin.scaled_zeros = torch.rand(lin.scaled_zeros.shape, generator=g).half()
    lin.bias = torch.rand(N, generator=g).half()
    return lin


@pytest.mark.parametrize("rows", [1, 3, 7])
def test_few_rows_reach_the_gemv_entry_point(ref_qmodule, rows):
    mod, calls = ref_qmodule
    lin = _ref_linear(mod)
    x = torch.randn(rows, 1024).half()
    out = lin(x)
    assert len(calls) == 1
    name, a = calls[0]
    assert name == "qvggt_w4a16_gemv"
    # (x, qweight, scales, scaled_zeros, bias, out, m, n, k, gpad, group_size, stream)
    assert _ptr(a[0]) == x.data_ptr()
    assert _ptr(a[1]) == lin.qweight.data_ptr()
    assert _ptr(a[2]) == lin.scales.data_ptr()
    assert _ptr(a[3]) == lin.scaled_zeros.data_ptr()
    assert a[4] is None                        # the reference adds the bias itself afterwards
    assert tuple(a[6:11]) == (rows, 512, 1024, lin.scales.shape[0], 128)
    assert out.shape == (rows, 512)


@pytest.mark.parametrize("rows,entry", [(8, "qvggt_small_linear"), (256, "qvggt_small_linear"),
                                        (300, "qvggt_w4a16_gemm")])
def test_more_rows_reach_the_gemm_entry_points(ref_qmodule, rows, entry):
    mod, calls = ref_qmodule
    lin = _ref_linear(mod)
    x = torch.randn(2, rows // 2, 1024).half()          # a leading batch dimension, as the aggregator passes
    out = lin(x)
    assert len(calls) == 1
    name, a = calls[0]
    assert name == entry
    M = x.numel() // 1024
    if entry == "qvggt_w4a16_gemm":
        # (x, qweight, scales, scaled_zeros, bias, out, M, N, K, gpad, group_size, stream)
        assert [_ptr(v) for v in a[:4]] == [x.data_ptr(), lin.qweight.data_ptr(), lin.scales.data_ptr(),
                                            lin.scaled_zeros.data_ptr()]
        assert a[4] is None
        assert tuple(a[6:11]) == (M, 512, 1024, lin.scales.shape[0], 128)
    else:
        # (kind, x, ldx, w, scales, zeros, gpad, group_size, bias, out, ldo, M, N, K, act, residual, ldr, gamma, stream)
        assert a[0] == 0
        assert _ptr(a[1]) == x.data_ptr() and a[2] == 1024
        assert [_ptr(v) for v in a[3:6]] == [lin.qweight.data_ptr(), lin.scales.data_ptr(),
                                             lin.scaled_zeros.data_ptr()]
        assert tuple(a[6:8]) == (lin.scales.shape[0], 128)
        assert a[8] is None
        assert tuple(a[11:15]) == (M, 512, 1024, 0)
    assert out.shape == (*x.shape[:-1], 512)


def test_reference_buffers_match_the_drop_in_buffers(ref_qmodule):
    """Same buffer names, shapes and dtypes, so ``model-v2.pt`` state dicts load into either."""
    from qvggt_b200 import qmodule
    mod, _ = ref_qmodule
    for K, N, G in ((1024, 3072, 128), (4096, 1024, 128), (2048, 8192, 128)):
        a = mod.WQLinear(4, G, K, N, True, "cpu").state_dict()
        b = qmodule.WQLinear(4, G, K, N, True, "cpu").state_dict()
        assert a.keys() == b.keys()
        for k in a:
            assert a[k].shape == b[k].shape and a[k].dtype == b[k].dtype, k
