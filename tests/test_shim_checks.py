"""Host-side argument checks of the drop-in shim (no GPU needed).

The kernels index raw device pointers, so every operand the shim hands to the
library must cover what the kernel reads or writes.  These tests drive the
shim's check helpers with CPU tensors of the shapes the public ops receive;
``tests/test_gpu_shape_errors.py`` calls the public ops themselves on a GPU.
"""
import pytest
import torch

from qvggt_b200 import awq_inference_engine as eng

F16 = torch.float16


def _w4(N=256, K=1024, G=128, gpad=8):
    return (torch.zeros(N // 4, K, dtype=torch.int16), torch.zeros(gpad, N, dtype=F16),
            torch.zeros(gpad, N, dtype=F16))


def test_w4_weights_accepts_the_reference_layout():
    qw, s, z = _w4()
    assert eng._check_w4_weights("t", qw, s, z, 1024, 128) == 256


@pytest.mark.parametrize("bad", ["qweight_k", "scales_n", "zeros_rows", "group", "dtype"])
def test_w4_weights_rejects_mismatched_buffers(bad):
    qw, s, z = _w4()
    K, G = 1024, 128
    if bad == "qweight_k":
        qw = torch.zeros(64, 512, dtype=torch.int16)
    elif bad == "scales_n":
        s = torch.zeros(8, 128, dtype=F16)
    elif bad == "zeros_rows":
        z = torch.zeros(4, 256, dtype=F16)          # K / G = 8 group rows needed
    elif bad == "group":
        G = 96
    elif bad == "dtype":
        s = s.float()
    with pytest.raises((ValueError, TypeError)):
        eng._check_w4_weights("t", qw, s, z, K, G)


def test_epilogue_checks():
    M, N = 5, 256
    eng._check_epilogue("t", M, N, bias=torch.zeros(N, dtype=F16), residual=torch.zeros(M, N, dtype=F16),
                        gamma=torch.zeros(N, dtype=F16))
    with pytest.raises(ValueError):
        eng._check_epilogue("t", M, N, bias=torch.zeros(N - 1, dtype=F16))
    with pytest.raises(ValueError):
        eng._check_epilogue("t", M, N, residual=torch.zeros(M + 1, N, dtype=F16))
    with pytest.raises(ValueError):      # a column slice is not contiguous: would be written in the wrong places
        eng._check_epilogue("t", M, N, out=torch.zeros(M, 2 * N, dtype=F16)[:, :N])
    with pytest.raises(TypeError):
        eng._check_epilogue("t", M, N, gamma=torch.zeros(N, dtype=torch.float32))


def test_row_operand_checks():
    q = torch.zeros(300, 3072, dtype=F16)
    eng._check_rows("t", q[:, :1024], 300, 1024, "q")          # a column view with unit column stride is fine
    with pytest.raises(ValueError):
        eng._check_rows("t", q[:, :1024], 301, 1024, "q")
    with pytest.raises(ValueError):
        eng._check_rows("t", q.t(), 300, 1024, "q")
    with pytest.raises(ValueError):
        eng._check_rows("t", q[:, :512], 300, 1024, "q")


def test_cpu_tensors_are_rejected_before_any_library_call():
    qw, s, z = _w4()
    with pytest.raises(ValueError, match="CUDA"):
        eng.gemm_forward_cuda_new(torch.zeros(3, 1024, dtype=F16), qw, s, z)
    with pytest.raises(ValueError, match="CUDA"):
        eng.w4a16_linear(torch.zeros(0, 1024, dtype=F16), qw, s, z)
