"""CPU: the PRODUCT packer (``qvggt_b200.qmodule``) against golden vectors made
by the reference's own Python code (``tests/golden/make_golden.py`` ran
``qvggt/runtime/awq/qmodule.py:43-99, 227-329`` on these inputs).

Every benchmarked and GPU-tested weight goes through these functions, so a
layout bug here would otherwise pass every kernel test (the kernels and the
oracle would read the same wrongly packed buffers) while disagreeing with
real ``model-v2.pt`` files.  Bit-exact.
"""
import numpy as np
import pytest
import torch
import torch.nn as nn

from qvggt_b200 import qmodule


def test_calculate_zeros_width_matches_reference(golden_pack):
    for K, G, w in golden_pack["czw"]:
        assert qmodule.calculate_zeros_width(int(K), int(G)) == int(w), (K, G)


@pytest.mark.parametrize("idx", range(5))
def test_pack_intweight_matches_reference(golden_pack, idx):
    """Including the inputs with values outside 0..15, which the reference
    ORs unmasked into neighbouring nibbles."""
    q = torch.from_numpy(golden_pack[f"pack{idx}_in"])
    mine = qmodule.pack_intweight(q)
    assert mine.dtype == torch.int16
    assert np.array_equal(mine.numpy(), golden_pack[f"pack{idx}_out"])


@pytest.mark.parametrize("idx", range(4))
def test_from_linear_matches_reference(golden_pack, idx):
    g = golden_pack
    w = torch.from_numpy(g[f"lin{idx}_weight"])
    N, K = w.shape
    lin = nn.Linear(K, N, bias=True).half()
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(torch.from_numpy(g[f"lin{idx}_bias"]))
    G = int(g[f"lin{idx}_G"])
    wq = qmodule.WQLinear.from_linear(lin, 4, G, scales=torch.from_numpy(g[f"lin{idx}_scales_in"]),
                                      zeros=torch.from_numpy(g[f"lin{idx}_zeros_in"]))
    assert np.array_equal(wq.qweight.numpy(), g[f"lin{idx}_qweight"])
    assert np.array_equal(wq.scales.numpy(), g[f"lin{idx}_scales"])
    assert np.array_equal(wq.scaled_zeros.numpy(), g[f"lin{idx}_scaled_zeros"])
    assert np.array_equal(wq.bias.numpy(), g[f"lin{idx}_out_bias"])


@pytest.mark.parametrize("idx", range(4))
def test_init_only_buffers_match_reference_shapes(golden_pack, idx):
    g = golden_pack
    N, K = g[f"lin{idx}_weight"].shape
    G = int(g[f"lin{idx}_G"])
    wq = qmodule.WQLinear.from_linear(nn.Linear(K, N, bias=True).half(), 4, G, init_only=True)
    assert wq.qweight.shape == g[f"lin{idx}_qweight"].shape and wq.qweight.dtype == torch.int16
    assert wq.scales.shape == g[f"lin{idx}_scales"].shape and wq.scales.dtype == torch.float16
    assert wq.scaled_zeros.shape == g[f"lin{idx}_scaled_zeros"].shape


def test_synthetic_quantizer_packs_like_the_reference():
    """``synthetic.quantize_w4`` (the benchmark's weights) packs its integer
    weights with the same function; round-tripping through the oracle's
    independent unpacker recovers them."""
    from oracle import awq
    from qvggt_b200.synthetic import quantize_w4
    w = torch.randn(64, 256, generator=torch.Generator().manual_seed(0)) * 0.02
    qw, st, szt = quantize_w4(w, 128)
    q = awq.unpack_intweight(qw.numpy())
    assert q.min() >= 0 and q.max() <= 15
    assert np.array_equal(qmodule.pack_intweight(torch.from_numpy(q)).numpy(), qw.numpy())
    deq = awq.dequantize(qw.numpy(), st.numpy(), szt.numpy(), 128).astype(np.float32)
    s = np.repeat(st.numpy()[:2].T.astype(np.float32), 128, axis=1)
    assert np.abs(deq - w.numpy()).max() <= 0.51 * s.max() + 1e-3
