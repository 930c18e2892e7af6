"""CPU: the oracle's DINOv2 front against PyTorch's own operators.

The patch GEMM over ``oracle.model.patchify`` columns must be the 14x14
stride-14 convolution with the checkpoint's [C, 3, 14, 14] weight (the loader
flattens it in the same order), and the special-token assembly must follow
VGGT's rule (set 0 for the first frame of the sequence, set 1 otherwise).
"""
import torch
import torch.nn.functional as F

from oracle import model as om


def test_patch_gemm_equals_conv2d():
    g = torch.Generator().manual_seed(0)
    S, C, p = 2, 32, 14
    images = torch.rand(S, 3, 6 * p, 5 * p, generator=g).half()
    w = (torch.randn(C, 3, p, p, generator=g) * 0.05).half()
    b = (torch.randn(C, generator=g) * 0.1).half()
    cols = om.patchify(images, p)                                    # [S * 6 * 5, 588]
    gemm = cols.float() @ w.reshape(C, -1).float().t() + b.float()
    m = torch.tensor(om.IMAGENET_MEAN, dtype=torch.float16).float().view(1, 3, 1, 1)
    s = torch.tensor(om.IMAGENET_STD, dtype=torch.float16).float().view(1, 3, 1, 1)
    norm = ((images.float() - m).half().float() / s).half().float()
    conv = F.conv2d(norm, w.float(), b.float(), stride=p)             # [S, C, 6, 5]
    conv = conv.permute(0, 2, 3, 1).reshape(S * 30, C)
    assert torch.allclose(gemm, conv, atol=1e-4, rtol=1e-4)


def test_aggregator_tokens_special_sets():
    S, n, C = 3, 7, 4
    pe_out = torch.arange(S * (5 + n) * C, dtype=torch.float32).reshape(S, 5 + n, C).half()
    specials = torch.stack([torch.full((5, C), 1.0), torch.full((5, C), 2.0)]).half()
    x = om.aggregator_tokens(pe_out, specials, frame_offset=0)
    assert torch.equal(x[0, :5], specials[0]) and torch.equal(x[1, :5], specials[1])
    assert torch.equal(x[2, :5], specials[1])
    assert torch.equal(x[:, 5:], pe_out[:, 5:])
    y = om.aggregator_tokens(pe_out, specials, frame_offset=4)       # a later rank's shard: no frame 0
    assert torch.equal(y[0, :5], specials[1])


def test_patch_embed_forward_layout():
    """cls + pos[0], registers without a position, patches + their positions."""
    g = torch.Generator().manual_seed(1)
    C, p = 16, 14
    images = torch.rand(1, 3, 2 * p, 3 * p, generator=g).half()
    pe = dict(patch_w=torch.zeros(C, 588).half(), patch_b=torch.zeros(C).half(),
              cls=torch.full((C,), 0.5).half(), registers=torch.randn(4, C, generator=g).half(),
              pos_cls=torch.full((C,), 0.25).half(), pos_patch=torch.randn(6, C, generator=g).half(),
              blocks=[], norm_w=torch.ones(C).half(), norm_b=torch.zeros(C).half(), patch=p)
    out = om.patch_embed_forward(images, pe, heads=1)
    ref = torch.cat([torch.full((1, C), 0.75), pe["registers"].float(), pe["pos_patch"].float()])
    assert torch.equal(out[0], om.layernorm(ref.half()[None], pe["norm_w"], pe["norm_b"])[0])
