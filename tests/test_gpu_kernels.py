"""GPU parity: W4A16 GEMM / GEMV, W8A8 chain, LayerNorm, RoPE kernels vs the CPU oracle.

Tolerances (stated per test): bit-exact for the int4 dequantisation and the
int32 accumulators; max-abs-rel <= 1e-2 per linear (fp32 oracle); int8
quantisation outputs within 1 code of the oracle on a tiny fraction of
elements (the reference itself uses approximate rsqrt / division there).
"""
import numpy as np
import pytest
import torch

from oracle import awq, model as om, rope as orope, w8a8 as ow

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from qvggt_b200 import _lib as L
    L.load()
    torch.manual_seed(0)
    yield


def _lin(N, K, G, seed):
    lin = awq.make_quantized_linear(N, K, G, seed=seed)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(DEV) for k, v in lin.items()
         if k in ("qweight", "scales", "scaled_zeros", "bias")}
    return lin, t


# ------------------------------------------------------------------ W4A16 GEMM
@pytest.mark.parametrize("M,N,K,G", [
    (1374, 4096, 1024, 128),   # BASELINE config 0 (fc1)
    (1374, 1024, 4096, 128),   # fc2 shape
    (300, 3072, 1024, 128),    # qkv shape, ragged M
    (129, 384, 256, 64),       # N % 256 != 0 -> 128-wide tiles, G = 64
    (17, 128, 128, 128),
    (2048, 256, 512, 128),
])
def test_w4a16_gemm_matches_oracle(M, N, K, G):
    from qvggt_b200 import awq_inference_engine as eng
    lin, t = _lin(N, K, G, seed=M + N)
    x = torch.randn(M, K, dtype=torch.float16)
    y = eng.gemm_forward_cuda_new(x.to(DEV), t["qweight"], t["scales"], t["scaled_zeros"], group_size=G)
    ref = awq.w4a16_linear(x, lin["qweight"], lin["scales"], lin["scaled_zeros"], G)
    err = awq.max_abs_rel(y.cpu(), ref)
    assert err <= 1e-2, err           # per-linear bound (fp32-accumulated oracle)
    assert err <= 2e-3, err           # what fp32 accumulation + one fp16 rounding gives


def test_w4a16_dequant_bit_exact_via_identity():
    """A = identity rows => C = deq(W)^T exactly (one non-zero term per sum)."""
    from qvggt_b200 import awq_inference_engine as eng
    N, K, G = 512, 256, 128
    lin, t = _lin(N, K, G, seed=7)
    eye = torch.eye(K, dtype=torch.float16, device=DEV)
    y = eng.gemm_forward_cuda_new(eye, t["qweight"], t["scales"], t["scaled_zeros"], group_size=G)
    deq = awq.dequantize(lin["qweight"], lin["scales"], lin["scaled_zeros"], G)   # [N, K]
    assert np.array_equal(y.cpu().numpy().T.view(np.uint16), deq.view(np.uint16))


def test_w4a16_dequant_all_nibbles_edge_scales_bit_exact():
    """Every nibble value under edge-case scales (subnormal, large) through the GEMM."""
    from qvggt_b200 import awq_inference_engine as eng
    N, K, G = 128, 128, 128
    q = np.tile(np.arange(16, dtype=np.int32), (N, K // 16))
    scales = np.array([1.0, 0.5, 2 ** -14, 2 ** -24, 65504 / 32, 0.0999755859375, 1e-3, 3.0] * 16, np.float16)
    zeros = (np.arange(N) % 16).astype(np.float32)
    st = np.zeros((8, N), np.float16)
    st[0] = scales
    szt = np.zeros((8, N), np.float16)
    szt[0] = (-(scales.astype(np.float32) * zeros)).astype(np.float16)
    qw = awq.pack_intweight(q)
    eye = torch.eye(K, dtype=torch.float16, device=DEV)
    y = eng.gemm_forward_cuda_new(eye, torch.from_numpy(qw).to(DEV), torch.from_numpy(st).to(DEV),
                                  torch.from_numpy(szt).to(DEV), group_size=G)
    deq = awq.dequantize(qw, st, szt, G)
    assert np.array_equal(y.cpu().numpy().T.view(np.uint16), deq.view(np.uint16))


@pytest.mark.parametrize("m", [1, 2, 7, 8, 16])
@pytest.mark.parametrize("N,K,G", [(4096, 1024, 128), (1024, 4096, 128), (256, 512, 32)])
def test_w4a16_gemv_matches_oracle(m, N, K, G):
    from qvggt_b200 import awq_inference_engine as eng
    lin, t = _lin(N, K, G, seed=m)
    x = torch.randn(m, K, dtype=torch.float16)
    y = eng.gemv_forward_cuda_new(x.to(DEV), t["qweight"], t["scales"], t["scaled_zeros"], m, N, K, G)
    ref = awq.w4a16_linear(x, lin["qweight"], lin["scales"], lin["scaled_zeros"], G)
    assert awq.max_abs_rel(y.cpu(), ref) <= 2e-3


def test_w4a16_gemv_dequant_bit_exact():
    from qvggt_b200 import awq_inference_engine as eng
    N, K, G = 256, 128, 64
    lin, t = _lin(N, K, G, seed=11)
    deq = awq.dequantize(lin["qweight"], lin["scales"], lin["scaled_zeros"], G)
    eye = torch.eye(K, dtype=torch.float16)
    for r0 in range(0, K, 16):
        y = eng.gemv_forward_cuda_new(eye[r0:r0 + 16].contiguous().to(DEV), t["qweight"], t["scales"],
                                      t["scaled_zeros"], 16, N, K, G)
        assert np.array_equal(y.cpu().numpy().T.view(np.uint16), deq[:, r0:r0 + 16].view(np.uint16))


def test_wqlinear_forward_bias_semantics():
    """WQLinear.forward = half(half(x W^T) + bias) through both GEMM and GEMV."""
    from qvggt_b200.qmodule import WQLinear
    N, K, G = 1024, 1024, 128
    lin, t = _lin(N, K, G, seed=5)
    m = WQLinear(4, G, K, N, True, DEV)
    m.qweight.copy_(t["qweight"]); m.scales.copy_(t["scales"]); m.scaled_zeros.copy_(t["scaled_zeros"])
    m.bias.copy_(t["bias"])
    for M in (3, 16, 17, 500):
        x = torch.randn(2, M, K, dtype=torch.float16)
        y = m(x.to(DEV)).cpu()
        assert y.shape == (2, M, N)
        ref = awq.wqlinear_forward_fp16(x, lin["qweight"], lin["scales"], lin["scaled_zeros"], G, lin["bias"])
        assert awq.max_abs_rel(y, ref) <= 2e-3


def test_fused_epilogues_gelu_and_residual():
    from qvggt_b200 import awq_inference_engine as eng
    N, K, G, M = 1024, 1024, 128, 777
    lin, t = _lin(N, K, G, seed=9)
    x = torch.randn(M, K, dtype=torch.float16)
    qlin = om.QLinear("w4", qweight=lin["qweight"], scales=lin["scales"], scaled_zeros=lin["scaled_zeros"],
                      bias=lin["bias"], group_size=G)
    y = eng.w4a16_linear(x.to(DEV), t["qweight"], t["scales"], t["scaled_zeros"], t["bias"], G, act="gelu").cpu()
    ref = om.gelu_erf(qlin(x))
    assert awq.max_abs_rel(y, ref) <= 2e-3
    resid = torch.randn(M, N, dtype=torch.float16)
    gamma = torch.full((N,), 0.37, dtype=torch.float16)
    r_dev = resid.to(DEV)
    eng.w4a16_linear(x.to(DEV), t["qweight"], t["scales"], t["scaled_zeros"], t["bias"], G, residual=r_dev,
                     gamma=gamma.to(DEV))
    ref2 = om.r16(resid.float() + om.r16(qlin(x).float() * gamma.float()).float())
    assert awq.max_abs_rel(r_dev.cpu(), ref2) <= 2e-3


def test_f16_linear_matches_oracle():
    from qvggt_b200 import awq_inference_engine as eng
    M, N, K = 1000, 1024, 640
    w = (torch.randn(N, K) * 0.02).half()
    b = (torch.randn(N) * 0.01).half()
    x = torch.randn(M, K, dtype=torch.float16)
    y = eng.f16_linear(x.to(DEV), w.to(DEV), b.to(DEV)).cpu()
    ref = om.QLinear("f16", weight=w, bias=b)(x)
    assert awq.max_abs_rel(y, ref) <= 2e-3


# ------------------------------------------------------------------------ W8A8
@pytest.mark.parametrize("M,N,K", [(1374, 4096, 1024), (300, 1024, 4096), (129, 384, 256), (5, 128, 128)])
def test_i8_gemm_accumulators_bit_exact(M, N, K):
    from qvggt_b200 import awq_inference_engine as eng
    g = torch.Generator().manual_seed(M)
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, generator=g)
    w = torch.randint(-128, 128, (N, K), dtype=torch.int8, generator=g)
    acc = eng.i8_gemm_i32(a.to(DEV), w.to(DEV)).cpu().numpy()
    assert np.array_equal(acc, ow.int8_gemm_i32(a.numpy(), w.numpy()))


@pytest.mark.parametrize("bias", [False, True])
def test_w8a8_gemm_epilogue(bias):
    from qvggt_b200 import awq_inference_engine as eng
    M, N, K = 513, 1024, 1024
    g = torch.Generator().manual_seed(3)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, generator=g)
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=g)
    ws = (torch.rand(N, generator=g) * 1e-3 + 1e-4).half()
    as_ = (torch.rand(M, generator=g) * 1e-2 + 1e-3).half()
    b = (torch.randn(N, generator=g) * 0.1).half()
    out = torch.empty(M, N, dtype=torch.float16, device=DEV)
    if bias:
        eng.w8a8_gemm_fuse_bias_forward_cuda(a.to(DEV), w.to(DEV), ws.to(DEV), as_.to(DEV), out, b.to(DEV))
        ref = ow.w8a8_gemm(a.numpy(), w.numpy(), ws.numpy(), as_.numpy(), b.numpy())
    else:
        eng.w8a8_gemm_forward_cuda(a.to(DEV), w.to(DEV), ws.to(DEV), as_.to(DEV), out)
        ref = ow.w8a8_gemm(a.numpy(), w.numpy(), ws.numpy(), as_.numpy())
    got = out.cpu().numpy()
    # identical fp32 operation sequence: equal up to rare 1-ulp double-rounding in the oracle
    mism = (got.view(np.uint16) != ref.view(np.uint16)).mean()
    assert mism < 1e-4, mism
    assert np.abs(got.astype(np.float32) - ref.astype(np.float32)).max() <= 2e-3 * np.abs(ref.astype(np.float32)).max()


def _int8_close(got, ref, frac=2e-3):
    d = np.abs(got.astype(np.int32) - ref.astype(np.int32))
    assert d.max() <= 1, d.max()
    assert (d > 0).mean() <= frac, (d > 0).mean()


def test_invoke_quant():
    from qvggt_b200 import awq_inference_engine as eng
    x = torch.randn(1000, 1024, dtype=torch.float16) * 3
    out = torch.empty(1000, 1024, dtype=torch.int8, device=DEV)
    sc = torch.empty(1000, dtype=torch.float16, device=DEV)
    eng.invoke_quant(out, x.to(DEV), sc)
    q, s = ow.invoke_quant(x.numpy())
    _int8_close(out.cpu().numpy(), q)
    assert np.array_equal(sc.cpu().numpy(), s)


@pytest.mark.parametrize("per_token", [True, False])
def test_rms_norm_general(per_token):
    from qvggt_b200 import awq_inference_engine as eng
    T, H = 777, 1024
    x = torch.randn(T, H, dtype=torch.float16) * 2 + 0.5
    w = (1 + 0.1 * torch.randn(H)).half()
    b = (0.1 * torch.randn(H)).half()
    out = torch.empty(T, H, dtype=torch.int8, device=DEV)
    if per_token:
        sc = torch.empty(T, dtype=torch.float16, device=DEV)
        eng.rms_norm_general(out, x.to(DEV), w.to(DEV), b.to(DEV), sc, 1e-6, True)
        q, s = ow.rms_norm_general(x.numpy(), w.numpy(), b.numpy(), 1e-6)
        _int8_close(out.cpu().numpy(), q)
        assert np.abs(sc.cpu().numpy().astype(np.float32) - s.astype(np.float32)).max() <= 1e-3 * np.abs(s).max()
    else:
        sc = torch.tensor([20.0], dtype=torch.float16, device=DEV)
        eng.rms_norm_general(out, x.to(DEV), w.to(DEV), b.to(DEV), sc, 1e-6, False)
        xf = x.float()
        mu = xf.mean(-1, keepdim=True)
        var = (xf * xf).mean(-1, keepdim=True) - mu * mu
        ln = ((xf - mu) * torch.rsqrt(var + 1e-6) * w.float()).half().float()
        q = ow.cvt_rni_sat_s8((ln * 20.0).numpy())
        _int8_close(out.cpu().numpy(), q, frac=5e-3)


def test_gelu_and_quant():
    from qvggt_b200 import awq_inference_engine as eng
    T, D = 500, 4096
    x = torch.randn(T, D, dtype=torch.float16) * 2
    out = torch.empty(T, D, dtype=torch.int8, device=DEV)
    sc = torch.empty(T, dtype=torch.float16, device=DEV)
    tmp = torch.empty(T, D, dtype=torch.float16, device=DEV)
    eng.gelu_and_quant(out, x.to(DEV), sc, tmp)
    q, s, t = ow.gelu_and_quant(x.numpy())
    tg = tmp.cpu().numpy()
    assert (tg.view(np.uint16) != t.view(np.uint16)).mean() < 1e-3          # tanhf vs float64 tanh
    assert np.abs(tg.astype(np.float32) - t.astype(np.float32)).max() <= 2e-3
    _int8_close(out.cpu().numpy(), q)
    assert np.abs(sc.cpu().numpy().astype(np.float32) - s.astype(np.float32)).max() <= 1e-3 * np.abs(s.astype(np.float32)).max()


def test_layernorm_fp16():
    from qvggt_b200 import awq_inference_engine as eng
    T, H = 3001, 1024
    x = torch.randn(T, H, dtype=torch.float16) * 3 + 1
    w = (1 + 0.1 * torch.randn(H)).half()
    b = (0.1 * torch.randn(H)).half()
    y = eng.layernorm(x.to(DEV), w.to(DEV), b.to(DEV), 1e-6).cpu()
    ref = om.layernorm(x, w, b, 1e-6)
    assert (y.float() - ref.float()).abs().max() <= 4e-3 * ref.float().abs().max()


# ------------------------------------------------------------------------ RoPE
@pytest.mark.parametrize("transpose", [False, True])
def test_fused_rope_with_pos(transpose):
    from qvggt_b200 import awq_inference_engine as eng
    s, b, h, d, d2 = 37, 3, 16, 64, 32
    x = torch.randn(b, s, h, d, dtype=torch.float16).transpose(0, 1)     # strided input
    freqs = torch.rand(b, s, d2) * 10
    y = eng.fused_rope_with_pos_forward_func(x.to(DEV), freqs.to(DEV), transpose)
    assert y.shape == (s, b, h, d)
    ref = orope.fused_rope_with_pos(x, freqs, transpose)
    assert (y.cpu().float() - ref.float()).abs().max() <= 4e-3
    if transpose:
        assert y.stride() == ref.stride()


@pytest.mark.parametrize("qk_norm", [False, True])
def test_qkv_rope2d(qk_norm):
    from qvggt_b200 import awq_inference_engine as eng
    S, P, H = 2, 1374, 16
    T = S * P
    qkv = torch.randn(T, 3 * H * 64, dtype=torch.float16)
    cos_t, sin_t = orope.rope2d_tables(64, 64)
    qn = None
    if qk_norm:
        qn = [(1 + 0.1 * torch.randn(64)).half(), (0.1 * torch.randn(64)).half(),
              (1 + 0.1 * torch.randn(64)).half(), (0.1 * torch.randn(64)).half()]
    q, kv = eng.qkv_rope2d(qkv.to(DEV), H, cos_t.to(DEV), sin_t.to(DEV), P, 5, 37,
                           qk_norm=None if qn is None else [t.to(DEV) for t in qn])
    pos = orope.patch_positions(P).repeat(S, 1)
    x = qkv.reshape(T, 3, H, 64).permute(1, 2, 0, 3)    # [3, H, T, 64]
    qr, kr = x[0], x[1]
    if qk_norm:
        qr = om.layernorm(qr, qn[0], qn[1], 1e-6)
        kr = om.layernorm(kr, qn[2], qn[3], 1e-6)
    qr = orope.rope2d(qr, pos).permute(1, 0, 2).reshape(T, H * 64)
    kr = orope.rope2d(kr, pos).permute(1, 0, 2).reshape(T, H * 64)
    tol = 4e-3 if qk_norm else 1e-3
    assert (q.cpu().float() - qr.float()).abs().max() <= tol
    assert (kv[:, : H * 64].cpu().float() - kr.float()).abs().max() <= tol
    assert torch.equal(kv[:, H * 64:].cpu(), qkv[:, 2 * H * 64:])


# ---------------------------------------------------------------- failure path
def test_bounded_wait_times_out_and_context_survives():
    import ctypes as C
    from qvggt_b200 import _lib as L
    st = C.c_uint32(0)
    rc = L.load().qvggt_selftest_wait_timeout(50_000_000, C.byref(st))
    assert rc == 4 and st.value == 0x1FF
    assert L.device_status(clear=True) == 0
    # the context is still usable
    test_w4a16_gemm_matches_oracle(300, 3072, 1024, 128)


def test_bad_arguments_raise():
    from qvggt_b200 import awq_inference_engine as eng
    from qvggt_b200._lib import QvggtError
    x = torch.randn(10, 100, dtype=torch.float16, device=DEV)
    qw = torch.zeros(32, 100, dtype=torch.int16, device=DEV)
    s = torch.zeros(8, 128, dtype=torch.float16, device=DEV)
    with pytest.raises((QvggtError, ValueError)):
        eng.gemm_forward_cuda_new(x, qw, s, s)          # K=100 not a multiple of 64 (nor of the group)
    with pytest.raises(ValueError):
        eng.gemm_forward_cuda_new(x.cpu(), qw, s, s)    # no CPU path
    with pytest.raises(RuntimeError):
        eng.gemv_forward_cuda_new(torch.zeros(17, 128, dtype=torch.float16, device=DEV), qw, s, s, 17, 128, 128, 128)


@pytest.mark.parametrize("kind,qk_norm", [("w4", False), ("w4", True), ("f16", False)])
def test_qkv_rope_linear_matches_separate_path(kind, qk_norm):
    """The qkv GEMM with the split + 2-D RoPE fused into its epilogue equals the
    separate GEMM(+bias) -> qkv_rope2d path bit for bit (same roundings)."""
    from qvggt_b200 import awq_inference_engine as eng
    from qvggt_b200.aggregator import AggConfig, rope_tables
    from qvggt_b200.synthetic import random_linear
    cfg = AggConfig()
    gen = torch.Generator(device=DEV).manual_seed(17)
    lin = random_linear(1024, 3072, gen, DEV, kind)
    T = 2 * 1374 + 100                                    # ragged: not a whole number of frames or tiles
    x = torch.randn(T, 1024, dtype=torch.float16, device=DEV)
    cos_t, sin_t = rope_tables(cfg, DEV)
    qn = None
    if qk_norm:
        qn = tuple(t.to(DEV) for t in ((1 + 0.1 * torch.randn(64)).half(), (0.1 * torch.randn(64)).half(),
                                       (1 + 0.1 * torch.randn(64)).half(), (0.1 * torch.randn(64)).half()))
    q1, kv1 = eng.qkv_rope_linear(x, lin, 16, cos_t, sin_t, qk_norm=qn)
    qkv = lin(x)
    q2, kv2 = eng.qkv_rope2d(qkv, 16, cos_t, sin_t, qk_norm=qn)
    assert torch.equal(q1, q2)
    assert torch.equal(kv1, kv2)


@pytest.mark.parametrize("mode", ["w4", "f16", "i8"])
def test_gemm_configs_agree_bit_for_bit(mode):
    """Every kernel configuration of the large-M GEMM (CTA pairs with 256-row
    tiles, 1-SM 128 x 256 and 128 x 128 tiles; ``qvggt_set_gemm_config``)
    accumulates each output over K in the same order, so all of them agree bit
    for bit, and with the oracle within the per-linear bound.  int8 has no pair
    form (that setting falls back to the automatic choice)."""
    from qvggt_b200 import _lib
    from qvggt_b200 import awq_inference_engine as eng
    M, N, K = 1000, 512, 1024     # ragged last row block
    g = torch.Generator().manual_seed(31)
    if mode == "i8":
        a = torch.randint(-128, 128, (M, K), dtype=torch.int8, generator=g).to(DEV)
        w = torch.randint(-128, 128, (N, K), dtype=torch.int8, generator=g).to(DEV)
        f = lambda: eng.i8_gemm_i32(a, w)
        ref = None
    else:
        x = torch.randn(M, K, generator=g).half().to(DEV)
        if mode == "w4":
            lin, t = _lin(N, K, 128, seed=3)
            f = lambda: eng.gemm_forward_cuda_new(x, t["qweight"], t["scales"], t["scaled_zeros"])
            ref = awq.w4a16_linear(x.cpu(), lin["qweight"], lin["scales"], lin["scaled_zeros"], 128)
        else:
            wt = (torch.randn(N, K, generator=g) * 0.02).half()
            f = lambda: eng.f16_linear(x, wt.to(DEV))
            ref = om.QLinear("f16", weight=wt, bias=None)(x.cpu()).float()
    outs = []
    try:
        for cfg in (1, 2, 3):
            _lib.call("qvggt_set_gemm_config", cfg)
            outs.append(f().clone())
    finally:
        _lib.call("qvggt_set_gemm_config", 0)
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    if mode == "i8":
        assert np.array_equal(outs[0].cpu().numpy(), ow.int8_gemm_i32(a.cpu().numpy(), w.cpu().numpy()))
    else:
        assert awq.max_abs_rel(outs[0].cpu(), ref) <= 2e-3


def test_gemm_config_choice():
    """The automatic choice keeps CTA pairs at the aggregator's full shapes and
    rejects an unknown setting."""
    from qvggt_b200 import _lib
    from qvggt_b200._lib import QvggtError
    with pytest.raises(QvggtError):
        _lib.call("qvggt_set_gemm_config", 7)


@pytest.mark.parametrize("M,N", [(4096, 4096), (10992, 3072)])
def test_w4_pair_gemm_equals_f16_pair_gemm_on_dequantised_weights(M, N):
    """The W4 pair kernel dequantises each CTA's half of B in shared memory and
    hands it to the pair MMA through a DSMEM bulk-copy signal; the fp16 pair
    kernel gets the same B halves by TMA.  With the exactly dequantised weights
    (fp16) the two must agree bit for bit, on every repetition (a stale B half
    would show up as a mismatch: a variant that split each k-block across all
    dequant warps failed here on the N = 3072 shape, in 32-channel blocks)."""
    from qvggt_b200 import awq_inference_engine as eng
    K, G = 1024, 128
    lin, t = _lin(N, K, G, seed=41)
    w16 = torch.from_numpy(awq.dequantize(lin["qweight"], lin["scales"], lin["scaled_zeros"], G)).half().to(DEV)
    g = torch.Generator().manual_seed(43)
    for _ in range(6):
        x = torch.randn(M, K, generator=g).half().to(DEV)
        y4 = eng.gemm_forward_cuda_new(x, t["qweight"], t["scales"], t["scaled_zeros"], group_size=G)
        y16 = eng.f16_linear(x, w16)
        assert torch.equal(y4, y16)


def test_w4_single_sm_gemm_equals_f16_on_dequantised_weights():
    """The 1-SM kernel (256 < M < 512 rows) dequantises through the same
    stage-release protocol as the pair kernel: bit-equal to the fp16 kernel on
    the exactly dequantised weights, on every repetition."""
    from qvggt_b200 import awq_inference_engine as eng
    M, N, K, G = 500, 3072, 1024, 128
    lin, t = _lin(N, K, G, seed=43)
    w16 = torch.from_numpy(awq.dequantize(lin["qweight"], lin["scales"], lin["scaled_zeros"], G)).half().to(DEV)
    g = torch.Generator().manual_seed(47)
    for _ in range(8):
        x = torch.randn(M, K, generator=g).half().to(DEV)
        y4 = eng.gemm_forward_cuda_new(x, t["qweight"], t["scales"], t["scaled_zeros"], group_size=G)
        assert torch.equal(y4, eng.f16_linear(x, w16))
