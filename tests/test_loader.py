"""Checkpoint loading (CPU): the reference loader's layout inference and
selective merge (``qvggt/inference/loader.py:164-224, 458-584``) restated in
``qvggt_b200.loader``, and a round trip aggregator -> state dict (VGGT key
layout) -> aggregator that must reproduce every weight bit for bit."""
import os
import tempfile
from collections import OrderedDict

import pytest
import torch

from qvggt_b200 import loader as L
from qvggt_b200.aggregator import AggConfig
from qvggt_b200.synthetic import random_vggt_aggregator


def _w4_keys(prefix):
    return {prefix + s: torch.zeros(1) for s in (".qweight", ".scales", ".scaled_zeros")}


def test_infer_quantization_layout():
    sd = {}
    sd.update(_w4_keys("aggregator.frame_blocks.0.attn.qkv"))
    sd.update(_w4_keys("aggregator.frame_blocks.2.mlp.fc1"))
    sd.update(_w4_keys("aggregator.global_blocks.1.attn.proj"))
    sd["aggregator.global_blocks.3.mlp.fc2.weight"] = torch.zeros(1)     # dense: not counted
    lay = L.infer_quantization_layout(sd)
    assert lay == {"frame_blocks": [0, 2], "global_blocks": [1], "quantize_camera_head": False,
                   "layer_types": ["fc1", "proj", "qkv"]}
    sd.update(_w4_keys("camera_head.trunk.0.attn.qkv"))
    assert L.infer_quantization_layout(sd)["quantize_camera_head"] is True
    assert L.infer_quantization_layout({"x.weight": torch.zeros(1)}) == {
        "frame_blocks": None, "global_blocks": None, "quantize_camera_head": False, "layer_types": None}


def test_merge_quantized_selects_blocks_and_drops_replaced_weights():
    orig = OrderedDict()
    for i in range(3):
        orig[f"aggregator.frame_blocks.{i}.attn.qkv.weight"] = torch.full((1,), float(i))
        orig[f"aggregator.frame_blocks.{i}.norm1.weight"] = torch.ones(1)
    q = OrderedDict(_w4_keys("aggregator.frame_blocks.1.attn.qkv"))
    q.update(_w4_keys("aggregator.frame_blocks.2.attn.qkv"))
    q["cict_token"] = torch.ones(3)
    q["unquantized_patch_start_idx"] = torch.tensor(5)
    with pytest.raises(ValueError):
        L.merge_quantized(q, None, frame_blocks=[1])
    merged, cict = L.merge_quantized(q, orig, frame_blocks=[1])
    assert torch.equal(cict, torch.ones(3))
    assert "aggregator.frame_blocks.1.attn.qkv.qweight" in merged
    assert "aggregator.frame_blocks.1.attn.qkv.weight" not in merged          # replaced
    assert "aggregator.frame_blocks.2.attn.qkv.weight" in merged              # block 2 not selected
    assert "aggregator.frame_blocks.2.attn.qkv.qweight" not in merged
    assert "cict_token" not in merged and "unquantized_patch_start_idx" not in merged
    merged_all, _ = L.merge_quantized(q, orig, quantize_type="all")
    assert "aggregator.frame_blocks.2.attn.qkv.weight" not in merged_all
    # a layer-type filter keeps the dense weight of other types
    merged_fc, _ = L.merge_quantized(q, orig, quantize_type="all", layer_types=["fc1"])
    assert "aggregator.frame_blocks.1.attn.qkv.weight" in merged_fc


def _small_cfg():
    return AggConfig(dim=128, heads=2, depth=2, qk_norm=True)


def _tensors_equal(a, b):
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b)


def _blocks_equal(x, y):
    for f in ("norm1_w", "norm1_b", "ls1", "norm2_w", "norm2_b", "ls2"):
        assert _tensors_equal(getattr(x, f), getattr(y, f)), f
    for f in ("qkv", "proj", "fc1", "fc2"):
        lx, ly = getattr(x, f), getattr(y, f)
        assert lx.kind == ly.kind
        names = ("qweight", "scales", "scaled_zeros") if lx.kind == "w4" else ("weight",)
        for n in names:
            assert _tensors_equal(getattr(lx, n), getattr(ly, n)), (f, n)
        assert (lx.bias is None) == (ly.bias is None)
        if lx.bias is not None:
            assert _tensors_equal(lx.bias, ly.bias)
    assert (x.qk_norm is None) == (y.qk_norm is None)
    if x.qk_norm is not None:
        assert all(_tensors_equal(a, b) for a, b in zip(x.qk_norm, y.qk_norm))


def test_state_dict_round_trip_cpu():
    cfg = _small_cfg()
    agg = random_vggt_aggregator(cfg, 3, "cpu", 1, pe_depth=2)
    sd = L.state_dict_from_aggregator(agg)
    assert sd["aggregator.camera_token"].shape == (1, 2, 1, 128)
    assert sd["aggregator.register_token"].shape == (1, 2, 4, 128)
    assert sd["aggregator.patch_embed.pos_embed"].shape == (1, 1 + 37 * 37, 128)
    assert L.infer_quantization_layout(sd)["frame_blocks"] == [0, 1]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "ckpt.pt")
        torch.save(OrderedDict(("model." + k, v) for k, v in sd.items()), path)   # wrapper prefix
        # not self-contained (no camera head): merged over the same dict as the fp16 base
        with pytest.raises(ValueError):
            L.load_aggregator(path, 1, "cpu", cfg=cfg)
        fp16 = os.path.join(d, "fp16.pt")
        torch.save(sd, fp16)
        agg2 = L.load_aggregator(path, 1, "cpu", original_path=fp16, cfg=cfg)
    pe, pe2 = agg.pe, agg2.pe
    for f in ("patch_w", "patch_b", "specials", "pos", "norm_w", "norm_b"):
        assert _tensors_equal(getattr(pe, f), getattr(pe2, f)), f
    assert len(pe.blocks) == len(pe2.blocks) == 2
    for x, y in zip(pe.blocks, pe2.blocks):
        _blocks_equal(x, y)
    for x, y in zip(agg.runner.frame_blocks + agg.runner.global_blocks,
                    agg2.runner.frame_blocks + agg2.runner.global_blocks):
        _blocks_equal(x, y)
    assert _tensors_equal(agg.agg_specials, agg2.agg_specials)


def test_missing_or_gapped_blocks_raise():
    cfg = _small_cfg()
    agg = random_vggt_aggregator(cfg, 4, "cpu", 1, pe_depth=1)
    sd = L.state_dict_from_aggregator(agg)
    gap = OrderedDict((k, v) for k, v in sd.items() if not k.startswith("aggregator.frame_blocks.0."))
    with pytest.raises(KeyError):
        L.aggregator_from_state_dict(gap, 1, "cpu", cfg=cfg)


def test_camera_trunk_round_trip_cpu():
    from qvggt_b200.camera_trunk import CameraTrunk
    from qvggt_b200.synthetic import random_block
    gen = torch.Generator().manual_seed(9)
    cfg = AggConfig(dim=256, heads=2)
    trunk = CameraTrunk([random_block(cfg, gen, "cpu", "w4") for _ in range(2)])
    sd = L.state_dict_from_camera_trunk(trunk)
    assert L.infer_quantization_layout(sd)["quantize_camera_head"] is True
    t2 = L.camera_trunk_from_state_dict(OrderedDict(("model." + k, v) for k, v in sd.items()), "cpu")
    assert len(t2.blocks) == 2
    for x, y in zip(trunk.blocks, t2.blocks):
        _blocks_equal(x, y)
