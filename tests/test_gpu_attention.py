"""GPU parity: tcgen05 flash attention (head_dim 64) vs the fp32 CPU oracle.

Tolerance: P is rounded to fp16 before the P.V product (as every fp16 flash
attention does) and O is rounded to fp16, so we require relative L2 <= 4e-3
and max-abs error <= 1.5e-2 * max|O_ref| for unit-scale inputs.
"""
import pytest
import torch

from oracle import awq, model as om

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(batches, Lq, Lkv, heads, qscale=1.0, seed=0):
    from qvggt_b200 import awq_inference_engine as eng
    g = torch.Generator().manual_seed(seed)
    C = heads * 64
    q = (torch.randn(batches * Lq, C, generator=g) * qscale).half()
    kv = torch.randn(batches * Lkv, 2 * C, generator=g).half()
    out = eng.attention(q.to(DEV), kv.to(DEV), heads, batches, Lq, Lkv).cpu()
    qh = q.reshape(batches, Lq, heads, 64).permute(0, 2, 1, 3)
    kh = kv[:, :C].reshape(batches, Lkv, heads, 64).permute(0, 2, 1, 3)
    vh = kv[:, C:].reshape(batches, Lkv, heads, 64).permute(0, 2, 1, 3)
    ref = om.sdpa(qh, kh, vh).permute(0, 2, 1, 3).reshape(batches * Lq, C)
    return out, ref


@pytest.mark.parametrize("batches,Lq,Lkv,heads", [
    (1, 128, 128, 1),
    (2, 300, 300, 2),       # ragged tiles
    (2, 1374, 1374, 16),    # frame attention, 2 frames
    (1, 2748, 2748, 16),    # global attention over 2 frames
    (3, 77, 1000, 4),       # Lq != Lkv, Lq < one tile
    (1, 256, 1, 2),         # single key
])
def test_attention_matches_oracle(batches, Lq, Lkv, heads):
    out, ref = _run(batches, Lq, Lkv, heads)
    assert torch.isfinite(out).all()
    assert awq.rel_l2(out, ref) <= 4e-3
    assert (out.float() - ref.float()).abs().max() <= 1.5e-2 * ref.float().abs().max()


def test_attention_large_scores_rescale_path():
    """Scores spanning a wide range force the running-max rescale of O."""
    out, ref = _run(1, 512, 2048, 2, qscale=6.0, seed=3)
    assert torch.isfinite(out).all()
    assert awq.rel_l2(out, ref) <= 4e-3


def test_attention_strided_views():
    """q / k / v read straight out of a packed qkv buffer [T, 3C]."""
    from qvggt_b200 import awq_inference_engine as eng
    heads, L = 4, 700
    C = heads * 64
    qkv = torch.randn(L, 3 * C).half()
    d = qkv.to(DEV)
    out = eng.attention(d[:, :C], d, heads, 1, L, L, k_col0=C, v_col0=2 * C).cpu()
    qh = qkv[:, :C].reshape(1, L, heads, 64).permute(0, 2, 1, 3)
    kh = qkv[:, C:2 * C].reshape(1, L, heads, 64).permute(0, 2, 1, 3)
    vh = qkv[:, 2 * C:].reshape(1, L, heads, 64).permute(0, 2, 1, 3)
    ref = om.sdpa(qh, kh, vh).permute(0, 2, 1, 3).reshape(L, C)
    assert awq.rel_l2(out, ref) <= 4e-3


def test_attention_repeatable_bit_for_bit():
    """Every output element is reduced in one fixed order (one CTA per query
    block, KV tiles in sequence), so repeated calls agree bit for bit; a race
    between the warp roles (an S, P or O buffer used before its hand-off)
    would show up as a difference between calls."""
    from qvggt_b200 import awq_inference_engine as eng
    g = torch.Generator(device=DEV).manual_seed(5)
    batches, L, heads = 1, 8192, 16
    q = torch.randn(batches * L, heads * 64, generator=g, device=DEV).half()
    kv = torch.randn(batches * L, 2 * heads * 64, generator=g, device=DEV).half()
    first = eng.attention(q, kv, heads, batches, L, L)
    for _ in range(8):
        assert torch.equal(eng.attention(q, kv, heads, batches, L, L), first)
