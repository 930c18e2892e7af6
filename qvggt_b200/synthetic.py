"""Seeded synthetic weights and inputs of the VGGT-1B architecture.

There is no checkpoint (the reference ships none), so benchmarks and tests
use random-init ``nn.Linear``-style weights N(0, 0.02), quantised the AWQ way
(asymmetric per group of 128 along K: s = (max - min) / 15, z = round(-min / s),
q = clamp(round(w / s + z), 0, 15)) and packed with
:func:`qvggt_b200.qmodule.pack_intweight`.  Generation runs on the target
device with a seeded torch generator.
"""
from __future__ import annotations

import torch

from .aggregator import AggConfig, Block, Linear
from .qmodule import calculate_zeros_width, pack_intweight

F16 = torch.float16


def quantize_w4(w: torch.Tensor, group_size: int = 128):
    """w [N, K] float -> (qweight int16 [N/4, K], scales fp16 [gpad, N], scaled_zeros fp16 [gpad, N])."""
    N, K = w.shape
    G = group_size
    wg = w.float().view(N, K // G, G)
    mx, mn = wg.amax(-1), wg.amin(-1)
    s = ((mx - mn) / 15.0).clamp_min(1e-5).to(F16)
    z = torch.round(-mn / s.float()).clamp(0, 15)
    q = torch.round(wg / s.float()[..., None] + z[..., None]).clamp(0, 15).to(torch.int32).view(N, K)
    gpad = calculate_zeros_width(K, G) * 8
    st = torch.zeros(gpad, N, dtype=F16, device=w.device)
    st[: K // G] = s.t()
    szt = torch.zeros(gpad, N, dtype=F16, device=w.device)
    szt[: K // G] = (-(s.float() * z)).to(F16).t()
    return pack_intweight(q), st.contiguous(), szt.contiguous()


def random_linear(K: int, N: int, gen: torch.Generator, device, kind: str = "w4", std: float = 0.02,
                  group_size: int = 128) -> Linear:
    w = torch.randn(N, K, generator=gen, device=device) * std
    bias = (torch.randn(N, generator=gen, device=device) * 0.01).to(F16)
    if kind == "w4":
        qw, st, szt = quantize_w4(w, group_size)
        return Linear("w4", bias, group_size, qweight=qw, scales=st, scaled_zeros=szt)
    if kind == "w8":
        # int8 symmetric per output channel, scale = max|W| / 127
        s = (w.abs().amax(dim=1) / 127.0).to(F16)
        q = torch.round(w / s.float()[:, None]).clamp(-128, 127).to(torch.int8).contiguous()
        return Linear("w8", bias, w8=q, wscale=s.contiguous())
    return Linear("f16", bias, weight=w.to(F16).contiguous())


def random_block(cfg: AggConfig, gen: torch.Generator, device, kind: str = "w4", layer_scale: float | None = None,
                 qk_norm: bool | None = None) -> Block:
    """One random-init block; ``qk_norm`` (default ``cfg.qk_norm``) adds the
    per-head q / k LayerNorm weights."""
    C = cfg.dim
    hd = C // cfg.heads
    ls = cfg.layer_scale if layer_scale is None else layer_scale
    r = lambda *shape: torch.randn(*shape, generator=gen, device=device)
    qn = None
    if cfg.qk_norm if qk_norm is None else qk_norm:
        qn = tuple(t.to(F16) for t in (1 + 0.1 * r(hd), 0.1 * r(hd), 1 + 0.1 * r(hd), 0.1 * r(hd)))
    return Block(
        norm1_w=(1 + 0.1 * r(C)).to(F16), norm1_b=(0.1 * r(C)).to(F16),
        qkv=random_linear(C, 3 * C, gen, device, kind, group_size=cfg.group_size),
        proj=random_linear(C, C, gen, device, kind, group_size=cfg.group_size),
        ls1=torch.full((C,), ls, dtype=F16, device=device),
        norm2_w=(1 + 0.1 * r(C)).to(F16), norm2_b=(0.1 * r(C)).to(F16),
        fc1=random_linear(C, cfg.mlp_ratio * C, gen, device, kind, group_size=cfg.group_size),
        fc2=random_linear(cfg.mlp_ratio * C, C, gen, device, kind, group_size=cfg.group_size),
        ls2=torch.full((C,), ls, dtype=F16, device=device),
        qk_norm=qn,
    )


def random_aggregator_blocks(cfg: AggConfig, seed: int, device, depth: int | None = None, kind: str = "w4"):
    gen = torch.Generator(device=device).manual_seed(seed)
    d = cfg.depth if depth is None else depth
    frame = [random_block(cfg, gen, device, kind) for _ in range(d)]
    glob = [random_block(cfg, gen, device, kind) for _ in range(d)]
    return frame, glob


def random_patch_embed(cfg: AggConfig, gen: torch.Generator, device, depth: int = 24, patch: int = 14,
                       k_pad: int = 640, layer_scale: float = 1e-5):
    """Random-init DINOv2 ViT-L/14-reg4 front (fp16, unquantised, no q/k norm),
    LayerScale 1e-5 as DINOv2 initialises it (tests raise it so the blocks'
    updates are not lost in the residual)."""
    from .aggregator import PatchEmbed
    C = cfg.dim
    kin = 3 * patch * patch
    w = torch.zeros(C, k_pad, device=device)
    w[:, :kin] = torch.randn(C, kin, generator=gen, device=device) * 0.02
    r = lambda *s: torch.randn(*s, generator=gen, device=device)
    pos = torch.zeros(cfg.tokens_per_frame, C, device=device)
    pos[0] = r(C) * 0.02
    pos[cfg.patch_start:] = r(cfg.tokens_per_frame - cfg.patch_start, C) * 0.02
    # the trained-table form [1 + M*M, C]: class position, then the patch grid
    pos_embed = torch.cat([pos[:1], pos[cfg.patch_start:]]).to(F16)
    blocks = [random_block(cfg, gen, device, kind="f16", layer_scale=layer_scale, qk_norm=False) for _ in range(depth)]
    return PatchEmbed(patch_w=w.to(F16).contiguous(), patch_b=(r(C) * 0.01).to(F16),
                      specials=(r(1, cfg.patch_start, C) * 0.02).to(F16).contiguous(), pos=pos.to(F16).contiguous(),
                      blocks=blocks, norm_w=(1 + 0.1 * r(C)).to(F16), norm_b=(0.1 * r(C)).to(F16), patch=patch,
                      k_pad=k_pad, pos_embed=pos_embed.cpu())


def random_vggt_aggregator(cfg: AggConfig, seed: int, device, frames_local: int, group=None, world: int = 1,
                           rank: int = 0, pe_depth: int = 24, kind: str = "w4", pe_layer_scale: float = 1e-5,
                           img_hw=(518, 518)):
    """Full synthetic VGGT-1B aggregator: DINOv2 front in fp16 + ``cfg.depth``
    frame/global pairs with ``kind`` linears ("w4": BASELINE config 2, "w8":
    the W8A8 chain of config 3), identical on every rank."""
    from .aggregator import VGGTAggregator
    gen = torch.Generator(device=device).manual_seed(seed)
    pe = random_patch_embed(cfg, gen, device, depth=pe_depth, layer_scale=pe_layer_scale)
    specials = (torch.randn(2, cfg.patch_start, cfg.dim, generator=gen, device=device) * 0.02).to(F16).contiguous()
    frame = [random_block(cfg, gen, device, kind) for _ in range(cfg.depth)]
    glob = [random_block(cfg, gen, device, kind) for _ in range(cfg.depth)]
    return VGGTAggregator(cfg, pe, specials, frame, glob, frames_local, device, group, world, rank, img_hw=img_hw)


def synthetic_images(S: int, seed: int, H: int = 518, W: int = 518) -> torch.Tensor:
    """RGB frames with pixels uniform in [0, 1] (CPU, fp16), BASELINE configs 2 / 4."""
    g = torch.Generator().manual_seed(seed)
    return torch.rand(S, 3, H, W, generator=g).to(F16)
