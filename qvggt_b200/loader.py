"""Loading a QVGGT checkpoint into the sm_100a runtime, without accelerate.

The checkpoint side restates the reference loader (``qvggt/inference/loader.py``):

* ``checkpoint_is_self_contained`` — ``loader.py:164-170``: a quantised
  checkpoint that also carries the patch embed, the aggregator's camera token
  and the camera head's pose branch needs no separate fp16 model.
* ``infer_quantization_layout`` — ``loader.py:178-224``: which frame / global
  blocks, which linear types (qkv / proj / fc1 / fc2) and whether the camera
  head trunk are quantised, read off the ``.qweight`` keys.
* ``merge_quantized`` — ``loader.py:458-584``: the auxiliary entries
  (``cict_token``, ``cict_topk``, ``unquantized_patch_start_idx``) are dropped,
  the selected quantised entries are laid over the fp16 state dict and every
  ``.weight`` they replace is removed.

The runtime side maps the merged state dict, keyed by the VGGT module tree
the checkpoints carry, onto this package's modules: ``aggregator.patch_embed.*``
(DINOv2 ViT-L/14 with 4 registers: ``patch_embed.proj``, ``cls_token``,
``register_tokens``, ``pos_embed``, ``blocks.N.*``, ``norm``) ->
:class:`~qvggt_b200.aggregator.PatchEmbed`; ``aggregator.frame_blocks.N.*`` and
``aggregator.global_blocks.N.*`` (``norm1``, ``attn.qkv``, ``attn.q_norm``,
``attn.k_norm``, ``attn.proj``, ``ls1.gamma``, ``norm2``, ``mlp.fc1``,
``mlp.fc2``, ``ls2.gamma``) -> :class:`~qvggt_b200.aggregator.Block`;
``aggregator.camera_token`` [1, 2, 1, C] and ``aggregator.register_token``
[1, 2, 4, C] -> the aggregator's special tokens; ``camera_head.trunk.N.*`` ->
:class:`~qvggt_b200.camera_trunk.CameraTrunk`.  A linear whose ``.qweight``,
``.scales`` and ``.scaled_zeros`` are present (the ``WQLinear`` buffers) runs
on the W4A16 kernels, one with a ``.weight`` on the dense fp16 kernels.
:func:`state_dict_from_aggregator` writes the same layout back (conversion,
round-trip tests).
"""
from __future__ import annotations

from collections import OrderedDict

import torch
import torch.nn.functional as Fnn

from .aggregator import AggConfig, Block, Linear, PatchEmbed, VGGTAggregator

F16 = torch.float16
AUX_KEYS = ("cict_token", "cict_topk", "unquantized_patch_start_idx")
SELF_CONTAINED_KEYS = ("aggregator.patch_embed.patch_embed.proj.weight", "aggregator.camera_token",
                       "camera_head.pose_branch.fc1.weight")
LAYER_TYPES = ("qkv", "proj", "fc1", "fc2")
W4_SUFFIXES = (".qweight", ".scales", ".scaled_zeros")


def _block_index(key: str, marker: str) -> int:
    return int(key.split(marker, 1)[1].split(".", 1)[0])


def strip_model_prefix(sd) -> OrderedDict:
    """Keys saved from a wrapper carry a leading ``model.`` (the reference
    also looks up ``model.camera_head.cict_token``, ``loader.py:226-234``)."""
    return OrderedDict((k[6:] if k.startswith("model.") else k, v) for k, v in sd.items())


def checkpoint_is_self_contained(sd) -> bool:
    return all(k in sd for k in SELF_CONTAINED_KEYS)


def infer_quantization_layout(sd) -> dict:
    """Quantised frame / global block indices, camera-head trunk flag and linear
    types, from the ``.qweight`` keys (None for an empty set, as the reference)."""
    frame, glob, types = set(), set(), set()
    camera = False
    for key in sd:
        if not key.endswith(".qweight"):
            continue
        if ".frame_blocks." in key:
            frame.add(_block_index(key, ".frame_blocks."))
        elif ".global_blocks." in key:
            glob.add(_block_index(key, ".global_blocks."))
        elif "camera_head.trunk." in key:
            camera = True
        types.update(t for t in LAYER_TYPES if f".{t}." in key)
    return {"frame_blocks": sorted(frame) or None, "global_blocks": sorted(glob) or None,
            "quantize_camera_head": camera, "layer_types": sorted(types) or None}


def merge_quantized(quantized_sd, original_sd=None, quantize_type: str = "specific_blocks", frame_blocks=None,
                    global_blocks=None, layer_types=None, quantize_camera_head: bool = True):
    """Lay the selected quantised entries over the fp16 state dict.

    Returns (merged state dict, cict_token or None).  A self-contained
    quantised checkpoint is its own base; otherwise ``original_sd`` (the fp16
    model) is required, as in the reference (ValueError without it).
    """
    q = OrderedDict(quantized_sd)
    cict = None
    for k in ("camera_head.cict_token", "model.camera_head.cict_token", "cict_token"):
        if k in q:
            cict = q[k]
            break
    for k in AUX_KEYS:
        q.pop(k, None)
    if checkpoint_is_self_contained(q):
        merged = OrderedDict(q)
    else:
        if original_sd is None:
            raise ValueError("checkpoint is not self-contained: the original fp16 state dict is required")
        merged = OrderedDict(original_sd)

    def layer_type(key):
        for t in LAYER_TYPES:
            if f".{t}" in key:
                return t
        return "linear" if "camera_head" in key else "unknown"

    def selected(key):
        if quantize_camera_head and "camera_head" in key:
            return True
        for marker, chosen in ((".frame_blocks.", frame_blocks), (".global_blocks.", global_blocks)):
            if marker in key:
                return quantize_type == "all" or (quantize_type == "specific_blocks" and chosen is not None
                                                  and _block_index(key, marker) in chosen)
        return False

    drop = set()
    for key, value in q.items():
        if not selected(key):
            continue
        if layer_types is not None and layer_type(key) not in layer_types:
            continue
        merged[key] = value
        for suf in W4_SUFFIXES:
            if key.endswith(suf):
                wkey = key[: -len(suf)] + ".weight"
                if wkey in merged and wkey != key:
                    drop.add(wkey)
    for k in drop:
        merged.pop(k, None)
    return merged, cict


# ---------------------------------------------------------------------- runtime modules
def _t(sd, key, device, dtype=None):
    v = sd[key]
    v = v.to(device)
    return v.to(dtype) if dtype is not None else v


def linear_from_state_dict(sd, prefix: str, device, group_size: int = 128) -> Linear:
    bias = _t(sd, prefix + ".bias", device, F16).contiguous() if prefix + ".bias" in sd else None
    if prefix + ".qweight" in sd:
        return Linear("w4", bias, group_size, qweight=_t(sd, prefix + ".qweight", device).contiguous(),
                      scales=_t(sd, prefix + ".scales", device, F16).contiguous(),
                      scaled_zeros=_t(sd, prefix + ".scaled_zeros", device, F16).contiguous())
    if prefix + ".weight" in sd:
        return Linear("f16", bias, weight=_t(sd, prefix + ".weight", device, F16).contiguous())
    raise KeyError(f"no weights for linear {prefix!r}")


def block_from_state_dict(sd, prefix: str, device, group_size: int = 128) -> Block:
    C = sd[prefix + ".norm1.weight"].shape[0]
    gamma = lambda name: (_t(sd, f"{prefix}.{name}.gamma", device, F16).contiguous()
                          if f"{prefix}.{name}.gamma" in sd else torch.ones(C, dtype=F16, device=device))
    qn = None
    if prefix + ".attn.q_norm.weight" in sd:
        qn = tuple(_t(sd, f"{prefix}.attn.{n}.{w}", device, F16).contiguous()
                   for n in ("q_norm", "k_norm") for w in ("weight", "bias"))
    return Block(
        norm1_w=_t(sd, prefix + ".norm1.weight", device, F16).contiguous(),
        norm1_b=_t(sd, prefix + ".norm1.bias", device, F16).contiguous(),
        qkv=linear_from_state_dict(sd, prefix + ".attn.qkv", device, group_size),
        proj=linear_from_state_dict(sd, prefix + ".attn.proj", device, group_size),
        ls1=gamma("ls1"),
        norm2_w=_t(sd, prefix + ".norm2.weight", device, F16).contiguous(),
        norm2_b=_t(sd, prefix + ".norm2.bias", device, F16).contiguous(),
        fc1=linear_from_state_dict(sd, prefix + ".mlp.fc1", device, group_size),
        fc2=linear_from_state_dict(sd, prefix + ".mlp.fc2", device, group_size),
        ls2=gamma("ls2"),
        qk_norm=qn,
    )


def _count(sd, prefix: str) -> int:
    idx = {_block_index(k, prefix) for k in sd if prefix in k}
    if idx and idx != set(range(len(idx))):
        raise KeyError(f"{prefix} indices are not contiguous: {sorted(idx)}")
    return len(idx)


def patch_embed_from_state_dict(sd, device, prefix: str = "aggregator.patch_embed", n_special: int = 5,
                                k_pad: int = 640) -> PatchEmbed:
    """DINOv2 front.  ``pos`` is the per-token table for the trained grid
    (37 x 37 patches, 518 x 518 frames, as VGGT's checkpoints store it); the
    trained table is kept as ``pos_embed`` so ``VGGTAggregator`` can resample
    it for other frame sizes."""
    w = sd[prefix + ".patch_embed.proj.weight"]                       # [C, 3, p, p]
    C, cin, p, _ = w.shape
    kin = cin * p * p
    if kin > k_pad:
        raise ValueError(f"patch of {kin} values exceeds k_pad={k_pad}")
    patch_w = Fnn.pad(w.reshape(C, kin).to(F16), (0, k_pad - kin)).to(device).contiguous()
    cls = sd[prefix + ".cls_token"].reshape(1, 1, C)
    regs = sd[prefix + ".register_tokens"].reshape(1, -1, C)
    if 1 + regs.shape[1] != n_special:
        raise ValueError(f"expected {n_special - 1} register tokens, got {regs.shape[1]}")
    pos_embed = sd[prefix + ".pos_embed"].reshape(-1, C)                 # [1 + M*M, C]
    pos = torch.zeros(pos_embed.shape[0] - 1 + n_special, C, dtype=F16)
    pos[0] = pos_embed[0].to(F16)
    pos[n_special:] = pos_embed[1:].to(F16)
    depth = _count(sd, prefix + ".blocks.")
    blocks = [block_from_state_dict(sd, f"{prefix}.blocks.{i}", device) for i in range(depth)]
    return PatchEmbed(patch_w=patch_w, patch_b=_t(sd, prefix + ".patch_embed.proj.bias", device, F16).contiguous(),
                      specials=torch.cat([cls, regs], 1).to(F16).to(device).contiguous(), pos=pos.to(device).contiguous(),
                      blocks=blocks, norm_w=_t(sd, prefix + ".norm.weight", device, F16).contiguous(),
                      norm_b=_t(sd, prefix + ".norm.bias", device, F16).contiguous(), patch=p, k_pad=k_pad,
                      pos_embed=pos_embed.detach().to(F16).cpu().contiguous())


def aggregator_from_state_dict(sd, frames_local: int, device, group=None, world: int = 1, rank: int = 0,
                               group_size: int = 128, cfg: AggConfig | None = None,
                               img_hw=(518, 518)) -> VGGTAggregator:
    """Build the runtime aggregator for this rank's ``frames_local`` frames of
    ``img_hw`` pixels (the position table is resampled for other sizes)."""
    sd = strip_model_prefix(sd)
    depth = _count(sd, "aggregator.frame_blocks.")
    if depth == 0 or depth != _count(sd, "aggregator.global_blocks."):
        raise KeyError("frame / global block counts are missing or differ")
    C = sd["aggregator.frame_blocks.0.norm1.weight"].shape[0]
    heads = (cfg.heads if cfg is not None else 16)
    if cfg is None:
        cfg = AggConfig(dim=C, heads=heads, depth=depth, group_size=group_size,
                        qk_norm="aggregator.frame_blocks.0.attn.q_norm.weight" in sd)
    frame = [block_from_state_dict(sd, f"aggregator.frame_blocks.{i}", device, group_size) for i in range(depth)]
    glob = [block_from_state_dict(sd, f"aggregator.global_blocks.{i}", device, group_size) for i in range(depth)]
    cam = sd["aggregator.camera_token"].reshape(2, 1, C)
    reg = sd["aggregator.register_token"].reshape(2, -1, C)
    specials = torch.cat([cam, reg], 1).to(F16).to(device).contiguous()          # [2, 5, C]
    pe = patch_embed_from_state_dict(sd, device, n_special=cfg.patch_start)
    return VGGTAggregator(cfg, pe, specials, frame, glob, frames_local, device, group, world, rank, img_hw=img_hw)


def camera_trunk_from_state_dict(sd, device, group_size: int = 128, prefix: str = "camera_head.trunk"):
    from .camera_trunk import CameraTrunk
    sd = strip_model_prefix(sd)
    depth = _count(sd, prefix + ".")
    return CameraTrunk([block_from_state_dict(sd, f"{prefix}.{i}", device, group_size) for i in range(depth)])


def load_aggregator(path: str, frames_local: int, device, original_path: str | None = None, **kw) -> VGGTAggregator:
    """``torch.load`` a checkpoint (merging it over an fp16 model when it is not
    self-contained, with the layout read off its ``.qweight`` keys) and build
    the runtime aggregator."""
    q = strip_model_prefix(torch.load(path, map_location="cpu"))
    lay = infer_quantization_layout(q)
    orig = strip_model_prefix(torch.load(original_path, map_location="cpu")) if original_path else None
    merged, _ = merge_quantized(q, orig, "specific_blocks", lay["frame_blocks"], lay["global_blocks"],
                                lay["layer_types"], lay["quantize_camera_head"])
    return aggregator_from_state_dict(merged, frames_local, device, **kw)


# ---------------------------------------------------------------------- export
def _put_linear(sd, prefix, lin: Linear):
    if lin.kind == "w4":
        sd[prefix + ".qweight"] = lin.qweight.cpu()
        sd[prefix + ".scales"] = lin.scales.cpu()
        sd[prefix + ".scaled_zeros"] = lin.scaled_zeros.cpu()
    elif lin.kind == "f16":
        sd[prefix + ".weight"] = lin.weight.cpu()
    else:
        raise NotImplementedError(f"export of {lin.kind} linears")
    if lin.bias is not None:
        sd[prefix + ".bias"] = lin.bias.cpu()


def _put_block(sd, prefix, b: Block):
    sd[prefix + ".norm1.weight"], sd[prefix + ".norm1.bias"] = b.norm1_w.cpu(), b.norm1_b.cpu()
    _put_linear(sd, prefix + ".attn.qkv", b.qkv)
    if b.qk_norm is not None:
        for (n, w), v in zip([(n, w) for n in ("q_norm", "k_norm") for w in ("weight", "bias")], b.qk_norm):
            sd[f"{prefix}.attn.{n}.{w}"] = v.cpu()
    _put_linear(sd, prefix + ".attn.proj", b.proj)
    sd[prefix + ".ls1.gamma"] = b.ls1.cpu()
    sd[prefix + ".norm2.weight"], sd[prefix + ".norm2.bias"] = b.norm2_w.cpu(), b.norm2_b.cpu()
    _put_linear(sd, prefix + ".mlp.fc1", b.fc1)
    _put_linear(sd, prefix + ".mlp.fc2", b.fc2)
    sd[prefix + ".ls2.gamma"] = b.ls2.cpu()


def state_dict_from_aggregator(agg: VGGTAggregator) -> OrderedDict:
    """The aggregator's weights under the checkpoint key layout above."""
    sd = OrderedDict()
    pe, cfg = agg.pe, agg.cfg
    C = cfg.dim
    kin = 3 * pe.patch * pe.patch
    p = "aggregator.patch_embed"
    sd[p + ".patch_embed.proj.weight"] = pe.patch_w[:, :kin].reshape(C, 3, pe.patch, pe.patch).cpu()
    sd[p + ".patch_embed.proj.bias"] = pe.patch_b.cpu()
    sd[p + ".cls_token"] = pe.specials[:, :1].cpu()
    sd[p + ".register_tokens"] = pe.specials[:, 1:].cpu()
    sd[p + ".pos_embed"] = torch.cat([pe.pos[:1], pe.pos[cfg.patch_start:]]).unsqueeze(0).cpu()
    for i, b in enumerate(pe.blocks):
        _put_block(sd, f"{p}.blocks.{i}", b)
    sd[p + ".norm.weight"], sd[p + ".norm.bias"] = pe.norm_w.cpu(), pe.norm_b.cpu()
    for i, b in enumerate(agg.runner.frame_blocks):
        _put_block(sd, f"aggregator.frame_blocks.{i}", b)
    for i, b in enumerate(agg.runner.global_blocks):
        _put_block(sd, f"aggregator.global_blocks.{i}", b)
    sd["aggregator.camera_token"] = agg.agg_specials[:, :1].reshape(1, 2, 1, C).cpu()
    sd["aggregator.register_token"] = agg.agg_specials[:, 1:].reshape(1, 2, -1, C).cpu()
    return sd


def state_dict_from_camera_trunk(trunk, prefix: str = "camera_head.trunk") -> OrderedDict:
    """The camera trunk's weights under ``camera_head.trunk.N.*``."""
    sd = OrderedDict()
    for i, b in enumerate(trunk.blocks):
        _put_block(sd, f"{prefix}.{i}", b)
    return sd
