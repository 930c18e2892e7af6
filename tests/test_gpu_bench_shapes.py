"""GPU parity at the shapes the benchmark times, against the CPU oracle.

* one frame/global block pair at S = 8 frames (global
  attention over T = 10,992 tokens), real dims (1024, 16 heads x 64, MLP 4096),
  W4A16 g128, q/k LayerNorm on, LayerScale 0.01.
* The global attention of config 2 (S = 32 on one GPU: Lq = Lkv = 43,968) and
  of config 4 on one of 8 GPUs (25 local frames against all 200: Lq = 34,350,
  Lkv = 274,800): the GPU computes every row; the fp32 oracle checks four
  64-row blocks spread over the queries (start, two interior, end) against
  all keys and all heads.
* The whole ``VGGTAggregator.forward`` (patchify, the patch GEMM, the position
  table, [cls | registers | patches] assembly, the DINOv2 blocks without RoPE,
  the final LayerNorm, the aggregator's camera / register tokens for frame 0
  against the other frames, then frame / global pairs) at real dims, S = 2,
  two DINOv2 blocks and two pairs, against ``oracle.model.aggregator_forward``.

Bounds: attention rel-L2 <= 4e-3 and max-abs <= 1.5e-2 * max|O| (as in
``test_gpu_attention.py``); block outputs rel-L2 <= 2e-2 (north-star e2e
bound), block updates rel-L2 <= 5e-2.
"""
import numpy as np
import pytest
import torch

from oracle import awq, model as om

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _oracle_block(blk) -> dict:
    from tests.test_gpu_aggregator import to_oracle_block
    return to_oracle_block(blk)


def test_config1_block_pair_s8_matches_oracle():
    from qvggt_b200.aggregator import AggConfig, AggregatorRunner
    from qvggt_b200.synthetic import random_block
    cfg = AggConfig()                                     # qk_norm on, LayerScale 0.01
    S, P, C = 8, cfg.tokens_per_frame, cfg.dim
    gen = torch.Generator(device=DEV).manual_seed(101)
    fb, gb = random_block(cfg, gen, DEV), random_block(cfg, gen, DEV)
    tokens = torch.randn(S, P, C, generator=torch.Generator().manual_seed(8)).half()
    run = AggregatorRunner(cfg, [fb], [gb], S, DEV)
    fr, gl = run.forward(tokens.to(DEV).clone())[-1]
    ref_f, ref_g = om.block_pair_forward(tokens, _oracle_block(fb), _oracle_block(gb))
    got_f, got_g = fr.view(S, P, C).cpu(), gl.view(S, P, C).cpu()
    assert awq.rel_l2(got_f, ref_f) <= 2e-2 and awq.rel_l2(got_g, ref_g) <= 2e-2
    assert awq.rel_l2(got_f.float() - tokens.float(), ref_f.float() - tokens.float()) <= 5e-2
    assert awq.rel_l2(got_g.float() - ref_f.float(), ref_g.float() - ref_f.float()) <= 5e-2


def _row_blocks(Lq: int, n: int = 64) -> list[int]:
    starts = [0, (Lq // 3) // n * n + 17, (2 * Lq // 3) // n * n + 5, Lq - n]
    return [r for s in starts for r in range(s, s + n)]


@pytest.mark.parametrize("Lq,Lkv", [(43968, 43968),       # config 2, one GPU
                                    (34350, 274800)])     # config 4, one rank of 8
def test_global_attention_bench_shape_row_subset(Lq, Lkv):
    from qvggt_b200 import awq_inference_engine as eng
    heads, C = 16, 1024
    g = torch.Generator(device=DEV).manual_seed(Lq)
    q = torch.randn(Lq, C, generator=g, device=DEV).half()
    kv = torch.randn(Lkv, 2 * C, generator=g, device=DEV).half()
    out = eng.attention(q, kv, heads, 1, Lq, Lkv)
    rows = torch.tensor(_row_blocks(Lq))
    got = out[rows.to(DEV)].cpu()
    kvc = kv.cpu()
    qh = q[rows.to(DEV)].cpu().reshape(1, -1, heads, 64).permute(0, 2, 1, 3)
    kh = kvc[:, :C].reshape(1, Lkv, heads, 64).permute(0, 2, 1, 3)
    vh = kvc[:, C:].reshape(1, Lkv, heads, 64).permute(0, 2, 1, 3)
    ref = om.sdpa(qh, kh, vh).permute(0, 2, 1, 3).reshape(-1, C)
    assert torch.isfinite(got.float()).all()
    assert awq.rel_l2(got, ref) <= 4e-3
    assert (got.float() - ref.float()).abs().max() <= 1.5e-2 * ref.float().abs().max()


def _oracle_patch_embed(pe, cfg) -> dict:
    k = 3 * pe.patch * pe.patch
    ps = cfg.patch_start
    return dict(patch_w=pe.patch_w[:, :k].cpu().numpy(), patch_b=pe.patch_b.cpu().numpy(),
                cls=pe.specials[0, 0].cpu(), registers=pe.specials[0, 1:ps].cpu(), pos_cls=pe.pos[0].cpu(),
                pos_patch=pe.pos[ps:].cpu(), blocks=[_oracle_block(b) for b in pe.blocks],
                norm_w=pe.norm_w.cpu(), norm_b=pe.norm_b.cpu(), patch=pe.patch)


def test_vggt_aggregator_forward_matches_oracle():
    from qvggt_b200.aggregator import AggConfig
    from qvggt_b200.synthetic import random_vggt_aggregator, synthetic_images
    cfg = AggConfig(depth=2, layer_scale=0.2)
    S = 2
    agg = random_vggt_aggregator(cfg, 23, DEV, S, pe_depth=2, pe_layer_scale=0.3)
    images = synthetic_images(S, 9)
    tokens = agg.embed(images.to(DEV)).clone().cpu()      # the aggregator's input, after the DINOv2 front
    fr, gl = agg.forward(images.to(DEV))[-1]
    pe = _oracle_patch_embed(agg.pe, cfg)
    x0, ref_f, ref_g = om.aggregator_forward(images, pe, agg.agg_specials.cpu(),
                                             [_oracle_block(b) for b in agg.runner.frame_blocks],
                                             [_oracle_block(b) for b in agg.runner.global_blocks])
    P, C = cfg.tokens_per_frame, cfg.dim
    # the front: camera / register rows exact (frame 0 gets set 0, frame 1 set 1), patch rows within tolerance
    assert torch.equal(tokens[:, :cfg.patch_start], x0[:, :cfg.patch_start])
    assert torch.equal(tokens[0, 0], agg.agg_specials[0, 0].cpu()) and torch.equal(tokens[1, 0],
                                                                                  agg.agg_specials[1, 0].cpu())
    assert awq.rel_l2(tokens[:, cfg.patch_start:], x0[:, cfg.patch_start:]) <= 2e-2
    got_f, got_g = fr.view(S, P, C).cpu(), gl.view(S, P, C).cpu()
    assert awq.rel_l2(got_f, ref_f) <= 2e-2
    assert awq.rel_l2(got_g, ref_g) <= 2e-2
    assert awq.rel_l2(got_g.float() - tokens.float(), ref_g.float() - x0.float()) <= 5e-2


def test_patchify_matches_oracle_bit_for_bit():
    """Normalisation and im2col of the patch embed: fp16 results identical."""
    from qvggt_b200 import awq_inference_engine as eng
    from qvggt_b200.synthetic import synthetic_images
    images = synthetic_images(3, 4)
    got = eng.patchify(images.to(DEV), 14, 640).cpu()
    ref = om.patchify(images, 14)
    assert torch.equal(got[:, :588], ref)
    assert not got[:, 588:].any()


def test_vggt_aggregator_landscape_frames_match_oracle():
    """Frames of 392 x 518 (QVGGT's crop of a 4:3 image: 28 x 37 patches,
    1,041 tokens per frame): the position table resampled from the trained
    37 x 37 one, the per-frame attention, the 2-D RoPE grid and the global
    attention follow the grid; against the oracle with its own resampling of
    the table."""
    from qvggt_b200.aggregator import AggConfig
    from qvggt_b200.synthetic import random_vggt_aggregator, synthetic_images
    H, W = 392, 518
    cfg = AggConfig(depth=1, layer_scale=0.2)
    S = 2
    agg = random_vggt_aggregator(cfg, 29, DEV, S, pe_depth=1, pe_layer_scale=0.3, img_hw=(H, W))
    assert agg.cfg.tokens_per_frame == 5 + 28 * 37 and agg.cfg.grid_w == 37
    images = synthetic_images(S, 12, H, W)
    tokens = agg.embed(images.to(DEV)).clone().cpu()
    fr, gl = agg.forward(images.to(DEV))[-1]
    pe = _oracle_patch_embed(agg.pe, agg.cfg)
    table = om.interpolate_pos_embed(agg.pe.pos_embed, 28, 37)
    pe["pos_cls"], pe["pos_patch"] = table[0].half(), table[1:].half()
    x0, ref_f, ref_g = om.aggregator_forward(images, pe, agg.agg_specials.cpu(),
                                             [_oracle_block(b) for b in agg.runner.frame_blocks],
                                             [_oracle_block(b) for b in agg.runner.global_blocks])
    P, C = agg.cfg.tokens_per_frame, agg.cfg.dim
    assert awq.rel_l2(tokens[:, 5:], x0[:, 5:]) <= 2e-2
    assert awq.rel_l2(fr.view(S, P, C).cpu(), ref_f) <= 2e-2
    assert awq.rel_l2(gl.view(S, P, C).cpu(), ref_g) <= 2e-2
    assert awq.rel_l2(gl.view(S, P, C).cpu().float() - tokens.float(), ref_g.float() - x0.float()) <= 5e-2
