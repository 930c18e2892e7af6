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


# ----------------------------------------------- segments, splits, log-sum-exp
def _qkv(batches, Lq, Lkv, heads, seed):
    g = torch.Generator().manual_seed(seed)
    C = heads * 64
    return (torch.randn(batches * Lq, C, generator=g).half(), torch.randn(batches * Lkv, 2 * C, generator=g).half())


def _oracle(q, kv, batches, Lq, Lkv, heads, rows=None):
    """fp32 attention (and natural log-sum-exp) over the key rows `rows` of each batch (default all)."""
    C = heads * 64
    qh = q.reshape(batches, Lq, heads, 64).permute(0, 2, 1, 3)
    kvb = kv.reshape(batches, Lkv, 2 * C)
    if rows is not None:
        kvb = kvb[:, rows]
    kh = kvb[..., :C].reshape(batches, -1, heads, 64).permute(0, 2, 1, 3)
    vh = kvb[..., C:].reshape(batches, -1, heads, 64).permute(0, 2, 1, 3)
    o, lse = om.sdpa_lse(qh, kh, vh)
    return o.permute(0, 2, 1, 3).reshape(batches * Lq, C), lse


@pytest.mark.parametrize("splits", [2, 3, 4])
@pytest.mark.parametrize("batches,Lq,Lkv,heads", [(1, 700, 3000, 4), (3, 300, 1374, 2)])
def test_attention_splits_match_oracle(splits, batches, Lq, Lkv, heads):
    from qvggt_b200 import awq_inference_engine as eng
    q, kv = _qkv(batches, Lq, Lkv, heads, 7)
    lse = torch.empty(batches, heads, Lq, dtype=torch.float32, device=DEV)
    out = eng.attention_ex(q.to(DEV), kv.to(DEV), heads, batches, Lq, Lkv, splits=splits, lse=lse, lse_mode=1).cpu()
    ref, ref_lse = _oracle(q, kv, batches, Lq, Lkv, heads)
    assert awq.rel_l2(out, ref) <= 4e-3
    assert (out.float() - ref.float()).abs().max() <= 1.5e-2 * ref.float().abs().max()
    assert (lse.cpu() - ref_lse).abs().max() <= 2e-3


@pytest.mark.parametrize("world,rank", [(2, 0), (3, 1), (4, 3)])
def test_attention_local_then_remote_merge(world, rank):
    """The split-pass global attention of a frame-sharded rank: its own key
    rows first (lse_mode 1), then the other ranks' rows in one or two
    segments (lse_mode 2) -- equal to one pass over all keys."""
    from qvggt_b200 import awq_inference_engine as eng
    from qvggt_b200.dist import remote_segments
    heads, T = 4, 1374
    q, kv = _qkv(1, T, T * world, heads, 11)
    qd, kvd = q.to(DEV), kv.to(DEV)
    lse = torch.empty(heads, T, dtype=torch.float32, device=DEV)
    out = torch.empty(T, heads * 64, dtype=torch.float16, device=DEV)
    eng.attention_ex(qd, kvd, heads, 1, T, T * world, out=out, segments=[(rank * T, T)], lse=lse, lse_mode=1)
    segs = remote_segments(T, world, rank)
    eng.attention_ex(qd, kvd, heads, 1, T, T * world, out=out, segments=segs, lse=lse, lse_mode=2)
    ref, ref_lse = _oracle(q, kv, 1, T, T * world, heads)
    got = out.cpu()
    assert awq.rel_l2(got, ref) <= 4e-3
    assert (got.float() - ref.float()).abs().max() <= 1.5e-2 * ref.float().abs().max()
    assert (lse.cpu() - ref_lse[0]).abs().max() <= 2e-3
    one = eng.attention(qd, kvd, heads, 1, T, T * world).cpu()
    assert awq.rel_l2(got, one) <= 2e-3


def test_attention_ragged_segments_batched():
    """Two segments per batch, neither starting nor ending on a 128-key tile,
    over three batches (frame-style), split in two."""
    from qvggt_b200 import awq_inference_engine as eng
    heads, Lq, Lkv = 2, 333, 1000
    q, kv = _qkv(3, Lq, Lkv, heads, 13)
    segs = [(37, 301), (500, 433)]
    rows = list(range(37, 338)) + list(range(500, 933))
    out = eng.attention_ex(q.to(DEV), kv.to(DEV), heads, 3, Lq, Lkv, segments=segs, splits=2).cpu()
    ref, _ = _oracle(q, kv, 3, Lq, Lkv, heads, rows)
    assert awq.rel_l2(out, ref) <= 4e-3


def test_attention_splits_repeatable_with_reused_scratch():
    """Consecutive split launches reuse one scratch buffer (its counters are
    cleared on the stream before each launch); the merge adds the splits in a
    fixed order, so results repeat bit for bit."""
    from qvggt_b200 import awq_inference_engine as eng
    heads, L = 16, 4096
    g = torch.Generator(device=DEV).manual_seed(3)
    q = torch.randn(L, heads * 64, generator=g, device=DEV).half()
    kv = torch.randn(L, 2 * heads * 64, generator=g, device=DEV).half()
    nbytes = eng.attention_scratch_bytes(1, L, heads, 3)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    first = eng.attention_ex(q, kv, heads, 1, L, L, splits=3, scratch=scratch).clone()
    for _ in range(6):
        assert torch.equal(eng.attention_ex(q, kv, heads, 1, L, L, splits=3, scratch=scratch), first)
    assert awq.rel_l2(first, eng.attention(q, kv, heads, 1, L, L)) <= 2e-3


def test_attention_plan_is_sane():
    from qvggt_b200 import awq_inference_engine as eng
    s1, b1 = eng.attention_plan(1, 43968, 43968, 16)
    assert s1 == 1 and b1 == 0                       # 2,752 items already fill the SMs in whole waves
    s8, b8 = eng.attention_plan(1, 5496, 5496 * 7, 16)
    assert 1 <= s8 <= 4 and (b8 > 0) == (s8 > 1)
    q, kv = (t.to(DEV) for t in _qkv(1, 256, 256, 1, 1))
    with pytest.raises(Exception, match="splits"):
        eng.attention_ex(q, kv, 1, 1, 256, 256, splits=5)
    with pytest.raises(Exception, match="splits"):
        eng.attention_ex(q, kv, 1, 1, 256, 256, splits=3)        # only 2 key tiles
