"""CPU: the AWQ oracle against golden vectors produced by the reference's own
Python packing code (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

from oracle import awq


def test_calculate_zeros_width(golden_pack):
    for K, G, w in golden_pack["czw"]:
        assert awq.calculate_zeros_width(int(K), int(G)) == int(w), (K, G)


@pytest.mark.parametrize("idx", range(5))
def test_pack_matches_reference(golden_pack, idx):
    q = golden_pack[f"pack{idx}_in"]
    ref = golden_pack[f"pack{idx}_out"]
    mine = awq.pack_intweight(q)
    assert mine.dtype == np.int16
    assert np.array_equal(mine, ref)
    if q.min() >= 0 and q.max() <= 15:
        assert np.array_equal(awq.unpack_intweight(ref), q)


@pytest.mark.parametrize("idx", range(4))
def test_from_linear_matches_reference(golden_pack, idx):
    g = golden_pack
    w = torch.from_numpy(g[f"lin{idx}_weight"])
    s = torch.from_numpy(g[f"lin{idx}_scales_in"])
    z = torch.from_numpy(g[f"lin{idx}_zeros_in"])
    G = int(g[f"lin{idx}_G"])
    qw, st, szt = awq.quantize_from_linear(w, s, z, G)
    assert np.array_equal(qw.numpy(), g[f"lin{idx}_qweight"])
    assert np.array_equal(st.numpy(), g[f"lin{idx}_scales"])
    assert np.array_equal(szt.numpy(), g[f"lin{idx}_scaled_zeros"])


@pytest.mark.parametrize("idx", range(4))
def test_dequant_reconstructs_weight(golden_pack, idx):
    """deq(q) = q*s - s*z approximates W to within half a quantisation step."""
    g = golden_pack
    G = int(g[f"lin{idx}_G"])
    w = g[f"lin{idx}_weight"].astype(np.float32)
    deq = awq.dequantize(g[f"lin{idx}_qweight"], g[f"lin{idx}_scales"], g[f"lin{idx}_scaled_zeros"], G)
    s = np.repeat(g[f"lin{idx}_scales_in"].astype(np.float32), G, axis=1)
    z = np.repeat(g[f"lin{idx}_zeros_in"].astype(np.float32), G, axis=1)
    wt = torch.from_numpy(g[f"lin{idx}_weight"])
    st16 = torch.from_numpy(g[f"lin{idx}_scales_in"])
    sz16 = torch.from_numpy(g[f"lin{idx}_zeros_in"]) * st16
    gi = torch.arange(wt.shape[1]) // G
    iw = torch.round((wt + sz16[:, gi]) / st16[:, gi]).numpy()   # fp16 math, as qmodule.py:289-309
    # The reference does not clamp or mask: an out-of-range value also corrupts
    # the other nibbles of its 16-bit word.  Skip every word that holds one.
    bad = ((iw < 0) | (iw > 15)).astype(np.int32)
    word_bad = awq.pack_intweight(bad).view(np.uint16) != 0          # [N/4, K] words
    ok = np.ones_like(bad, dtype=bool)
    N_, K_ = bad.shape
    for n in range(N_):
        for k in range(K_):
            c, r = divmod(k, 64)
            w_ = (r // 32) * 8 + (r % 8)
            if word_bad[n // 4, 64 * c + 16 * (n % 4) + w_]:
                ok[n, k] = False
    assert ok.mean() > 0.9
    err = np.abs(deq.astype(np.float32) - w)
    assert np.all(err[ok] <= (1.0 * s + 2e-3 * np.abs(w) + 1e-3)[ok])


def test_dequant_all_nibbles_kat():
    """Known answers: every nibble value 0..15 under edge scales, one fp16 rounding."""
    N, K, G = 16, 128, 128
    q = np.tile(np.arange(16, dtype=np.int32), (N, K // 16))
    scales = np.array([1.0, 0.5, 2 ** -14, 2 ** -24, 65504 / 16, 0.0999755859375, 1e-3, 3.0,
                       0.02, 7.5, 1 / 3, 2 ** -10, 0.25, 1.5, 100.0, 0.0078125], np.float16)
    zeros = np.arange(16, dtype=np.float32)
    st = np.zeros((8, N), np.float16)
    st[0] = scales
    szt = np.zeros((8, N), np.float16)
    szt[0] = (-(scales.astype(np.float32) * zeros)).astype(np.float16)
    deq = awq.dequantize(awq.pack_intweight(q), st, szt, G)
    exp = (q.astype(np.float64) * scales.astype(np.float64)[:, None]
           + szt[0].astype(np.float64)[:, None]).astype(np.float16)
    assert np.array_equal(deq.view(np.uint16), exp.view(np.uint16))


def test_linear_oracle_matches_dense():
    lin = awq.make_quantized_linear(256, 512, 128, seed=3)
    x = torch.randn(37, 512).half()
    y = awq.w4a16_linear(x, lin["qweight"], lin["scales"], lin["scaled_zeros"], 128, lin["bias"])
    w = torch.from_numpy(awq.dequantize(lin["qweight"], lin["scales"], lin["scaled_zeros"], 128)).double()
    y64 = x.double() @ w.t() + torch.from_numpy(lin["bias"]).double()
    assert awq.max_abs_rel(y, y64) < 1e-5
