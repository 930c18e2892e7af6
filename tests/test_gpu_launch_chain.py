"""GPU: long chains of dependent launches give the same bits whether the
kernels overlap or not.

Every kernel of the library is launched with programmatic dependent launch:
it may start while the kernel before it on the stream is still running and
must not touch global memory before that kernel has completed.  A kernel
that read its input too early would read a stale or half-written buffer.
Here a chain of a block's worth of kernels (LayerNorm -> fused qkv / RoPE
GEMM -> attention -> residual GEMM -> LayerNorm -> GELU GEMM -> residual
GEMM, plus the W4A16 pair kernel and the GEMV), each reading the previous
one's output, runs back to back several times, and again with a device
synchronisation after every launch (so nothing can overlap).  The results
must be identical bit for bit: the kernels are deterministic.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from qvggt_b200 import _lib as L
    L.load()
    yield


def _chain(x, p, rounds, sync):
    from qvggt_b200 import awq_inference_engine as eng
    T, C = x.shape
    h = torch.empty_like(x)
    q = torch.empty_like(x)
    kv = torch.empty(T, 2 * C, dtype=torch.float16, device=DEV)
    attn = torch.empty_like(x)
    mlp = torch.empty(T, 4 * C, dtype=torch.float16, device=DEV)
    s = (lambda: torch.cuda.synchronize()) if sync else (lambda: None)
    for _ in range(rounds):
        eng.layernorm(x, p["n1w"], p["n1b"], out=h); s()
        eng.qkv_rope_linear(h, p["qkv"], 16, p["cos"], p["sin"], tokens_per_frame=T // 2, q_out=q, kv_out=kv)
        s()
        eng.attention(q, kv, 16, 2, T // 2, T // 2, out=attn); s()
        eng.w4a16_linear(attn, *p["proj"], bias=p["pb"], residual=x, gamma=p["g1"]); s()
        eng.layernorm(x, p["n2w"], p["n2b"], out=h); s()
        eng.w4a16_linear(h, *p["fc1"], bias=p["f1b"], act="gelu", out=mlp); s()
        eng.w4a16_linear(mlp, *p["fc2"], bias=p["f2b"], residual=x, gamma=p["g2"]); s()
        y = eng.w4a16_linear(x[:2].contiguous(), *p["proj"], bias=p["pb"]); s()   # the GEMV
        x[:2].copy_(y); s()
    return x


def _params(C):
    from qvggt_b200.aggregator import AggConfig, rope_tables
    from qvggt_b200.synthetic import quantize_w4
    g = torch.Generator(device=DEV).manual_seed(5)
    rnd = lambda *sh, sc=1.0: (torch.randn(*sh, generator=g, device=DEV) * sc).half()
    w4 = lambda N, K: quantize_w4(torch.randn(N, K, generator=g, device=DEV) * 0.02, 128)

    class Lin:
        pass
    qkv = Lin()
    qkv.qweight, qkv.scales, qkv.scaled_zeros = w4(3 * C, C)
    qkv.bias = rnd(3 * C, sc=0.01)
    qkv.group_size = 128
    qkv.weight = None
    qkv.kind = "w4"
    cos, sin = rope_tables(AggConfig(), DEV)
    return dict(n1w=1 + rnd(C, sc=0.1), n1b=rnd(C, sc=0.1), n2w=1 + rnd(C, sc=0.1), n2b=rnd(C, sc=0.1),
                qkv=qkv, cos=cos, sin=sin, proj=w4(C, C), pb=rnd(C, sc=0.01),
                fc1=w4(4 * C, C), f1b=rnd(4 * C, sc=0.01), fc2=w4(C, 4 * C), f2b=rnd(C, sc=0.01),
                g1=rnd(C, sc=0.1), g2=rnd(C, sc=0.1))


def test_dependent_launch_chain_matches_synchronised_chain():
    C, T = 1024, 2 * 1374
    p = _params(C)
    x0 = (torch.randn(T, C, generator=torch.Generator(device=DEV).manual_seed(6), device=DEV)).half()
    a = _chain(x0.clone(), p, rounds=6, sync=False)
    torch.cuda.synchronize()
    b = _chain(x0.clone(), p, rounds=6, sync=True)
    assert torch.isfinite(a.float()).all()
    assert torch.equal(a, b)
