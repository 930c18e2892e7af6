"""The public ops reject operands that do not cover what the kernel would touch,
before anything is launched, and an empty input gives an empty result."""
import pytest
import torch

from qvggt_b200 import awq_inference_engine as eng

pytestmark = pytest.mark.gpu
F16 = torch.float16
DEV = "cuda"


def _w4(N=256, K=1024, gpad=8):
    return (torch.zeros(N // 4, K, dtype=torch.int16, device=DEV), torch.zeros(gpad, N, dtype=F16, device=DEV),
            torch.zeros(gpad, N, dtype=F16, device=DEV))


def test_w4_mismatched_scales_raise():
    qw, s, z = _w4()
    x = torch.zeros(600, 1024, dtype=F16, device=DEV)
    with pytest.raises(ValueError):
        eng.gemm_forward_cuda_new(x, qw, s[:, :128].contiguous(), z)
    with pytest.raises(ValueError):
        eng.w4a16_linear(x, qw, s, z[:4].contiguous())
    with pytest.raises(ValueError):
        eng.w4a16_linear(x, qw, s, z, bias=torch.zeros(100, dtype=F16, device=DEV))
    with pytest.raises(ValueError):
        eng.w4a16_linear(x, qw, s, z, residual=torch.zeros(600, 512, dtype=F16, device=DEV)[:, :256],
                         gamma=torch.zeros(256, dtype=F16, device=DEV))


def test_w8a8_mismatched_operands_raise():
    M, N, K = 300, 512, 1024
    a = torch.zeros(M, K, dtype=torch.int8, device=DEV)
    w = torch.zeros(N, K, dtype=torch.int8, device=DEV)
    ws = torch.ones(N, dtype=F16, device=DEV)
    as_ = torch.ones(M, dtype=F16, device=DEV)
    out = torch.empty(M, N, dtype=F16, device=DEV)
    eng.w8a8_gemm_forward_cuda(a, w, ws, as_, out)
    with pytest.raises(ValueError):
        eng.w8a8_gemm_forward_cuda(a, w[:, :512].contiguous(), ws, as_, out)
    with pytest.raises(ValueError):
        eng.w8a8_gemm_forward_cuda(a, w, ws[:10], as_, out)
    with pytest.raises(ValueError):
        eng.w8a8_gemm_forward_cuda(a, w, ws, as_[:10], out)
    with pytest.raises(TypeError):
        eng.w8a8_gemm_residual(a, w, ws, as_, None, torch.ones(N, dtype=F16, device=DEV),
                               torch.zeros(M, N, dtype=torch.float32, device=DEV))


def test_attention_short_operands_raise():
    q = torch.zeros(1000, 1024, dtype=F16, device=DEV)
    kv = torch.zeros(1000, 2048, dtype=F16, device=DEV)
    with pytest.raises(ValueError):
        eng.attention(q, kv, 16, 1, 1000, 1001)
    with pytest.raises(ValueError):
        eng.attention(q[:, :512], kv, 16, 1, 1000, 1000)


def test_empty_input_gives_empty_output():
    qw, s, z = _w4()
    x = torch.zeros(0, 1024, dtype=F16, device=DEV)
    assert eng.w4a16_linear(x, qw, s, z).shape == (0, 256)
    assert eng.gemm_forward_cuda_new(x, qw, s, z).shape == (0, 256)
    assert eng.f16_linear(x, torch.zeros(256, 1024, dtype=F16, device=DEV)).shape == (0, 256)
