"""VGGT aggregator forward on the sm_100a kernels.

The aggregator (defined in the un-vendored ``vggt-hf`` model the reference
loads at ``qvggt/inference/loader.py:27``) runs, after the DINOv2 patch embed,
24 alternating frame / global block pairs over tokens [S, P, C]
(P = 1 camera + 4 register + 37*37 patch tokens, C = 1024).  Each block is

    x += ls1 * proj(attn(rope2d(q), rope2d(k), v)),  q, k, v = qkv(LN1(x))
    x += ls2 * fc2(gelu(fc1(LN2(x))))

with the frame block attending within each frame and the global block over
all S*P tokens.  The reference quantises every qkv / proj / fc1 / fc2 of both
block types to W4A16 (``loader.py:320-394``).

Kernel sequence of one block (W4A16):

    layernorm -> W4 GEMM(qkv, +bias, q/k/v split + 2-D RoPE in the epilogue)
    -> flash attention -> W4 GEMM(proj, +bias, LayerScale residual, in place)
    -> layernorm -> W4 GEMM(fc1, +bias, GELU) -> W4 GEMM(fc2, +bias, LayerScale residual)

Multi-GPU: frames are sharded contiguously over ranks.  Frame blocks and all
linears are rank-local; a global block writes its roped K / V straight into
this rank's slice of a [S*P, 2C] buffer and starts the NCCL all-gather of the
buffer; while it is in flight the local queries attend to the rank's own keys
(writing the rows' log-sum-exp), then, once the gather has landed, to the
other ranks' keys, and the second pass merges the two results exactly.  No
other communication.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import awq_inference_engine as eng
from .dist import gather_kv, kv_slice, remote_segments

F16 = torch.float16


@dataclass
class AggConfig:
    dim: int = 1024
    heads: int = 16
    mlp_ratio: int = 4
    depth: int = 24                  # frame/global block pairs
    tokens_per_frame: int = 1374     # 1 camera + 4 register + 37*37 patches
    patch_start: int = 5
    grid_w: int = 37
    eps: float = 1e-6
    rope_base: float = 100.0
    # VGGT-1B's aggregator blocks LayerNorm q and k per head (over head_dim)
    # before RoPE; the DINOv2 front's blocks do not.
    qk_norm: bool = True
    group_size: int = 128
    layer_scale: float = 0.01


class Linear:
    """A linear in one of three forms, holding device buffers:
    ``w4`` (AWQ qweight / scales / scaled_zeros), ``f16`` (dense weight [N, K])."""

    def __init__(self, kind: str, bias: torch.Tensor | None, group_size: int = 128, **bufs):
        self.kind = kind
        self.bias = bias
        self.group_size = group_size
        for k, v in bufs.items():
            setattr(self, k, v)
        if kind == "w4":
            self.out_features = self.qweight.shape[0] * 4
            self.in_features = self.qweight.shape[1]
        elif kind == "w8":   # int8 weight [N, K] + fp16 per-channel scale `wscale` [N]
            self.out_features, self.in_features = self.w8.shape
        else:
            self.out_features, self.in_features = self.weight.shape

    @classmethod
    def from_oracle(cls, ql, device) -> "Linear":
        """From an ``oracle.model.QLinear``-like object holding numpy buffers."""
        t = lambda a: None if a is None else torch.as_tensor(np.ascontiguousarray(a)).to(device)
        if ql.kind == "w4":
            return cls("w4", t(ql.bias), ql.group_size, qweight=t(ql.qweight), scales=t(ql.scales),
                       scaled_zeros=t(ql.scaled_zeros))
        return cls("f16", t(ql.bias), weight=t(ql.weight))

    def __call__(self, x, out=None, act=None, residual=None, gamma=None):
        if self.kind == "w4":
            return eng.w4a16_linear(x, self.qweight, self.scales, self.scaled_zeros, self.bias, self.group_size,
                                    act=act, residual=residual, gamma=gamma, out=out)
        return eng.f16_linear(x, self.weight, self.bias, act=act, residual=residual, gamma=gamma, out=out)


@dataclass
class Block:
    norm1_w: torch.Tensor
    norm1_b: torch.Tensor
    qkv: Linear
    proj: Linear
    ls1: torch.Tensor
    norm2_w: torch.Tensor
    norm2_b: torch.Tensor
    fc1: Linear
    fc2: Linear
    ls2: torch.Tensor
    qk_norm: tuple | None = None

    @classmethod
    def from_oracle(cls, blk: dict, device) -> "Block":
        t = lambda a: torch.as_tensor(np.ascontiguousarray(a)).to(device)
        qn = None
        if blk.get("qk_norm"):
            qn = (t(blk["qn_w"]), t(blk["qn_b"]), t(blk["kn_w"]), t(blk["kn_b"]))
        return cls(t(blk["norm1_w"]), t(blk["norm1_b"]), Linear.from_oracle(blk["qkv"], device),
                   Linear.from_oracle(blk["proj"], device), t(blk["ls1"]), t(blk["norm2_w"]), t(blk["norm2_b"]),
                   Linear.from_oracle(blk["fc1"], device), Linear.from_oracle(blk["fc2"], device), t(blk["ls2"]), qn)


def rope_tables(cfg: AggConfig, device):
    """cos / sin [max_pos, head_dim/2] fp16, computed as the model does (fp32
    angles cast to fp16, then cos / sin rounded to fp16)."""
    hd = cfg.dim // cfg.heads
    f = hd // 2
    max_pos = (cfg.tokens_per_frame - cfg.patch_start + cfg.grid_w - 1) // cfg.grid_w + 2
    inv = 1.0 / (cfg.rope_base ** (torch.arange(0, f, 2, dtype=torch.float32) / f))
    ang = torch.einsum("i,j->ij", torch.arange(max_pos, dtype=torch.float32), inv).to(F16)
    ang = torch.cat([ang, ang], dim=-1).float()
    return ang.cos().to(F16).to(device).contiguous(), ang.sin().to(F16).to(device).contiguous()


class Workspace:
    """Activation buffers for T local tokens (allocated once, reused by every block)."""

    def __init__(self, T_local: int, T_global: int, cfg: AggConfig, device, w8a8: bool = False):
        C = cfg.dim
        if w8a8:   # int8 activations + per-token fp16 scales of the W8A8 chain
            self.xq = torch.empty(T_local, C, dtype=torch.int8, device=device)
            self.xs = torch.empty(T_local, dtype=F16, device=device)
            self.mq = torch.empty(T_local, cfg.mlp_ratio * C, dtype=torch.int8, device=device)
            self.ms = torch.empty(T_local, dtype=F16, device=device)
        self.h = torch.empty(T_local, C, dtype=F16, device=device)
        self.qkv = torch.empty(T_local, 3 * C, dtype=F16, device=device)
        self.q = torch.empty(T_local, C, dtype=F16, device=device)
        self.kv_local = torch.empty(T_local, 2 * C, dtype=F16, device=device)
        self.kv_global = torch.empty(T_global, 2 * C, dtype=F16, device=device)
        self.attn = torch.empty(T_local, C, dtype=F16, device=device)
        self.mlp = torch.empty(T_local, cfg.mlp_ratio * C, dtype=F16, device=device)
        # split-pass global attention (more than one rank): per-row log-sum-exp
        # and the kernels' split scratch
        self.lse = None
        self.attn_scratch = None
        if T_global > T_local:
            self.lse = torch.empty(cfg.heads, T_local, dtype=torch.float32, device=device)


class AggregatorRunner:
    """Runs the aggregator block stack for this rank's frames.

    ``frames_local`` frames of ``cfg.tokens_per_frame`` tokens live on this
    rank; ``group`` (a torch.distributed process group, or None for one GPU)
    provides the K/V all-gather of the global blocks.
    """

    def __init__(self, cfg: AggConfig, frame_blocks: list[Block], global_blocks: list[Block], frames_local: int,
                 device, group=None, world: int = 1, rank: int = 0, overlap_kv: bool = True):
        self.cfg = cfg
        self.frame_blocks = frame_blocks
        self.global_blocks = global_blocks
        self.S_local = frames_local
        self.world = world
        self.rank = rank
        self.group = group
        self.device = torch.device(device)
        P = cfg.tokens_per_frame
        self.T = frames_local * P
        self.w8a8 = any(b.qkv.kind == "w8" for b in list(frame_blocks) + list(global_blocks))
        self.ws = Workspace(self.T, self.T * world, cfg, self.device, self.w8a8)
        self.cos, self.sin = rope_tables(cfg, self.device)
        # With more than one rank the global attention runs as a local-keys
        # pass overlapping the K/V all-gather and a remote-keys pass
        # (overlap_kv), or after the whole gather (overlap_kv=False).
        # Every global attention uses the library's split plan (split-KV when
        # the local query blocks alone would leave a partial wave of CTAs).
        # (A runner built on the CPU, e.g. to load or save a checkpoint, keeps
        # one split: it never launches anything.)
        self.overlap_kv = overlap_kv and world > 1
        self.split_all = self.split_local = self.split_remote = 1
        b0 = b1 = b2 = 0
        if self.device.type == "cuda":
            with torch.cuda.device(self.device):
                self.split_all, b0 = eng.attention_plan(1, self.T, self.T * world, cfg.heads)
                self.split_local, b1 = eng.attention_plan(1, self.T, self.T, cfg.heads)
                if world > 1:
                    self.split_remote, b2 = eng.attention_plan(1, self.T, self.T * (world - 1), cfg.heads)
        if max(b0, b1, b2):
            self.ws.attn_scratch = torch.empty(max(b0, b1, b2), dtype=torch.uint8, device=self.device)
        # When a list: one dict per global-attention call, appended by the
        # global blocks: CUDA events ("passes": [(start, end), ...] around
        # each attention launch; "wait": (end of the local pass, gather landed)
        # with the split passes) and the algorithmic FLOP of the call.
        self.kernel_timer = None

    # ------------------------------------------------------------------ block
    def block(self, x: torch.Tensor, blk: Block, kind: str, rope: bool = True) -> None:
        """One block over x [T_local, C] in place.  ``rope=False`` (the DINOv2
        patch-embed blocks) attends within each frame straight out of the qkv
        buffer, without RoPE."""
        cfg, ws = self.cfg, self.ws
        P = cfg.tokens_per_frame
        C = cfg.dim
        if blk.qkv.kind == "w8":
            return self.block_w8a8(x, blk, kind)
        eng.layernorm(x, blk.norm1_w, blk.norm1_b, cfg.eps, out=ws.h)
        if not rope:
            blk.qkv(ws.h, out=ws.qkv)
            eng.attention(ws.qkv[:, :C], ws.qkv, cfg.heads, self.S_local, P, P, out=ws.attn, k_col0=C, v_col0=2 * C)
            blk.proj(ws.attn, residual=x, gamma=blk.ls1)
            eng.layernorm(x, blk.norm2_w, blk.norm2_b, cfg.eps, out=ws.h)
            blk.fc1(ws.h, out=ws.mlp, act="gelu")
            blk.fc2(ws.mlp, residual=x, gamma=blk.ls2)
            return
        glob = kind == "global"
        if glob and self.world > 1:
            kv_dst = kv_slice(ws.kv_global, self.T, self.rank)
        else:
            kv_dst = ws.kv_local
        # qkv projection with the q/k/v split and 2-D RoPE in the GEMM epilogue
        eng.qkv_rope_linear(ws.h, blk.qkv, cfg.heads, self.cos, self.sin, P, cfg.patch_start, cfg.grid_w, 0,
                            q_out=ws.q, kv_out=kv_dst, qk_norm=blk.qk_norm, eps=cfg.eps)
        if glob:
            self._global_attention()
        else:
            eng.attention(ws.q, ws.kv_local, cfg.heads, self.S_local, P, P, out=ws.attn)
        blk.proj(ws.attn, residual=x, gamma=blk.ls1)
        eng.layernorm(x, blk.norm2_w, blk.norm2_b, cfg.eps, out=ws.h)
        blk.fc1(ws.h, out=ws.mlp, act="gelu")
        blk.fc2(ws.mlp, residual=x, gamma=blk.ls2)

    def _global_attention(self) -> None:
        """Attention of the local queries (``ws.q``) over every frame's keys
        into ``ws.attn``; this rank's roped K / V are in its slice of
        ``ws.kv_global`` (world > 1) or in ``ws.kv_local``."""
        cfg, ws, T = self.cfg, self.ws, self.T
        timer = self.kernel_timer
        ev = (lambda: torch.cuda.Event(enable_timing=True)) if timer is not None else None
        if self.world == 1 or not self.overlap_kv:
            if self.world > 1:
                kv, Lkv = gather_kv(ws.kv_global, T, self.rank, self.group), T * self.world
            else:
                kv, Lkv = ws.kv_local, T
            e = [ev(), ev()] if timer is not None else None
            if e:
                e[0].record()
            eng.attention_ex(ws.q, kv, cfg.heads, 1, T, Lkv, out=ws.attn, splits=self.split_all,
                             scratch=ws.attn_scratch)
            if e:
                e[1].record()
                timer.append({"passes": [(e[0], e[1])], "flop": 4.0 * T * Lkv * cfg.dim})
            return
        Lkv = T * self.world
        work = gather_kv(ws.kv_global, T, self.rank, self.group, async_op=True)
        e = [ev() for _ in range(4)] if timer is not None else None
        if e:
            e[0].record()
        eng.attention_ex(ws.q, ws.kv_global, cfg.heads, 1, T, Lkv, out=ws.attn, segments=[(self.rank * T, T)],
                         splits=self.split_local, lse=ws.lse, lse_mode=1, scratch=ws.attn_scratch)
        if e:
            e[1].record()
        work.wait()
        if e:
            e[2].record()
        eng.attention_ex(ws.q, ws.kv_global, cfg.heads, 1, T, Lkv, out=ws.attn,
                         segments=remote_segments(T, self.world, self.rank), splits=self.split_remote, lse=ws.lse,
                         lse_mode=2, scratch=ws.attn_scratch)
        if e:
            e[3].record()
            timer.append({"passes": [(e[0], e[1]), (e[2], e[3])], "wait": (e[1], e[2]),
                          "flop": 4.0 * T * Lkv * cfg.dim})

    def _attend(self, kind: str, kv_dst: torch.Tensor) -> None:
        cfg, ws = self.cfg, self.ws
        if kind == "global":
            self._global_attention()
        else:
            eng.attention(ws.q, ws.kv_local, cfg.heads, self.S_local, cfg.tokens_per_frame, cfg.tokens_per_frame,
                          out=ws.attn)

    def block_w8a8(self, x: torch.Tensor, blk: Block, kind: str) -> None:
        """W8A8 block, the chain the reference's W8A8 ops
        imply: LayerNorm + per-token int8 (rms_norm_general) -> int8 GEMM
        (+bias) -> 2-D RoPE -> attention -> per-token int8 (invoke_quant) ->
        int8 GEMM (+bias, LayerScale residual) -> LayerNorm + int8 -> int8 GEMM
        (+bias) -> tanh-GELU + int8 (gelu_and_quant) -> int8 GEMM (+bias,
        LayerScale residual)."""
        cfg, ws = self.cfg, self.ws
        P = cfg.tokens_per_frame
        eng.rms_norm_general(ws.xq, x, blk.norm1_w, blk.norm1_b, ws.xs, cfg.eps, True)
        q = blk.qkv
        eng.w8a8_gemm_fuse_bias_forward_cuda(ws.xq, q.w8, q.wscale, ws.xs, ws.qkv, q.bias)
        glob = kind == "global"
        kv_dst = kv_slice(ws.kv_global, self.T, self.rank) if (glob and self.world > 1) else ws.kv_local
        eng.qkv_rope2d(ws.qkv, cfg.heads, self.cos, self.sin, P, cfg.patch_start, cfg.grid_w, 0, q_out=ws.q,
                       kv_out=kv_dst, qk_norm=blk.qk_norm, eps=cfg.eps)
        self._attend(kind, kv_dst)
        eng.invoke_quant(ws.xq, ws.attn, ws.xs)
        eng.w8a8_gemm_residual(ws.xq, blk.proj.w8, blk.proj.wscale, ws.xs, blk.proj.bias, blk.ls1, x)
        eng.rms_norm_general(ws.xq, x, blk.norm2_w, blk.norm2_b, ws.xs, cfg.eps, True)
        eng.w8a8_gemm_fuse_bias_forward_cuda(ws.xq, blk.fc1.w8, blk.fc1.wscale, ws.xs, ws.mlp, blk.fc1.bias)
        eng.gelu_and_quant(ws.mq, ws.mlp, ws.ms, ws.mlp)          # tmp written in place over the fc1 output
        eng.w8a8_gemm_residual(ws.mq, blk.fc2.w8, blk.fc2.wscale, ws.ms, blk.fc2.bias, blk.ls2, x)

    def forward(self, tokens: torch.Tensor, keep: tuple[int, ...] = ()) -> dict:
        """tokens [S_local, P, C] fp16 (modified in place).  Runs every pair;
        returns {layer: (frame_out, global_out)} copies for the pair indices in
        ``keep`` plus the final pair under key -1."""
        x = tokens.view(self.T, self.cfg.dim)
        outs = {}
        n = len(self.frame_blocks)
        for i in range(n):
            self.block(x, self.frame_blocks[i], "frame")
            fr = x.clone() if (i in keep or i == n - 1) else None
            self.block(x, self.global_blocks[i], "global")
            if fr is not None:
                outs[-1 if i == n - 1 else i] = (fr, x.clone())
        return outs



@dataclass
class PatchEmbed:
    """DINOv2 ViT-L/14 with 4 registers (the aggregator's fp16, unquantised
    front; excluded from quantisation at ``loader.py:346``)."""
    patch_w: torch.Tensor      # [C, k_pad] fp16, column c*p*p + ky*p + kx, zero padded
    patch_b: torch.Tensor      # [C]
    specials: torch.Tensor     # [1, 5, C]: cls then 4 register tokens
    pos: torch.Tensor          # [P, C]: pos[0] for cls, 0 for registers, pos[1+i] for patch i
    blocks: list               # Block (kind f16), no RoPE
    norm_w: torch.Tensor
    norm_b: torch.Tensor
    patch: int = 14
    k_pad: int = 640
    # the trained position table [1 + M*M, C] (class position, M x M patch
    # grid), kept to build `pos` for other frame sizes; None: `pos` only
    pos_embed: torch.Tensor | None = None


class VGGTAggregator:
    """Images [S_local, 3, H, W] -> aggregator outputs, on this rank's frames.

    patchify -> patch GEMM -> [cls | registers | patches] + pos -> DINOv2 blocks
    -> LayerNorm -> [camera | registers | patch tokens] (first frame of the
    sequence uses its own camera / register tokens) -> 24 frame/global pairs.

    ``img_hw``: the frame size, multiples of the patch size (QVGGT's loader
    gives 518 wide and at most 518 tall, ``qvggt_b200.frames.crop_size``).  A
    patch grid other than the position table's is served with the table
    resampled to it (``frames.token_position_table``); the token count per
    frame, the 2-D RoPE grid width and the frame attention follow the grid.
    """

    def __init__(self, cfg: AggConfig, pe: PatchEmbed, agg_specials: torch.Tensor, frame_blocks, global_blocks,
                 frames_local: int, device, group=None, world: int = 1, rank: int = 0, img_hw=(518, 518)):
        import dataclasses
        H, W = img_hw
        if H <= 0 or W <= 0 or H % pe.patch or W % pe.patch:
            raise ValueError(f"frame size {img_hw} must be positive multiples of the patch size {pe.patch}")
        rows, cols = H // pe.patch, W // pe.patch
        self.n_patch = rows * cols
        if self.n_patch + cfg.patch_start != cfg.tokens_per_frame or cols != cfg.grid_w:
            cfg = dataclasses.replace(cfg, tokens_per_frame=self.n_patch + cfg.patch_start, grid_w=cols)
        if pe.pos.shape[0] != cfg.tokens_per_frame:
            if pe.pos_embed is None:
                raise ValueError(f"the position table holds {pe.pos.shape[0] - cfg.patch_start} patches, the "
                                 f"{H} x {W} frames have {self.n_patch}, and no trained table to resample")
            from .frames import token_position_table
            pos = token_position_table(pe.pos_embed, rows, cols, cfg.patch_start)
            pe = dataclasses.replace(pe, pos=pos.to(pe.pos.device).contiguous())
        self.cfg = cfg
        self.pe = pe
        self.agg_specials = agg_specials            # [2, 5, C]: camera + 4 registers, frame 0 / others
        self.runner = AggregatorRunner(cfg, frame_blocks, global_blocks, frames_local, device, group, world, rank)
        self.S_local = frames_local
        self.rank = rank
        self.img_hw = img_hw
        dev = torch.device(device)
        C = cfg.dim
        self.patches = torch.empty(frames_local * self.n_patch, pe.k_pad, dtype=F16, device=dev)
        self.pe_out = torch.empty(frames_local * self.n_patch, C, dtype=F16, device=dev)
        self.x_pe = torch.empty(frames_local, cfg.tokens_per_frame, C, dtype=F16, device=dev)
        self.tokens = torch.empty(frames_local, cfg.tokens_per_frame, C, dtype=F16, device=dev)

    def forward(self, images: torch.Tensor, keep: tuple[int, ...] = ()) -> dict:
        """The DINOv2 front, then the frame / global pairs (which update
        ``self.tokens`` in place); returns the runner's outputs."""
        return self.runner.forward(self.embed(images), keep)

    def embed(self, images: torch.Tensor) -> torch.Tensor:
        """images [S_local, 3, H, W] -> the aggregator's input tokens
        ``self.tokens`` [S_local, P, C]: DINOv2 front, final LayerNorm, then
        camera / register tokens in place of DINOv2's special rows."""
        cfg, pe = self.cfg, self.pe
        P, C = cfg.tokens_per_frame, cfg.dim
        eng.patchify(images, pe.patch, pe.k_pad, out=self.patches)
        eng.f16_linear(self.patches, pe.patch_w, pe.patch_b, out=self.pe_out)
        eng.assemble_tokens(self.pe_out, self.n_patch, 0, pe.specials, cfg.patch_start, False, pe.pos, self.x_pe,
                            self.S_local, P)
        x = self.x_pe.view(-1, C)
        for blk in pe.blocks:
            self.runner.block(x, blk, "frame", rope=False)
        h = self.runner.ws.h
        eng.layernorm(x, pe.norm_w, pe.norm_b, cfg.eps, out=h)
        eng.assemble_tokens(h, P, cfg.patch_start, self.agg_specials, cfg.patch_start, True, None, self.tokens,
                            self.S_local, P, frame_offset=self.rank * self.S_local)
        return self.tokens

    def infer(self, images_host: torch.Tensor, out_host: torch.Tensor | None = None):
        """Public end-to-end call: host images [S_local, 3, H, W] fp16 (pinned
        for asynchronous copies) -> host tensor [S_local, P, 2C] holding the
        last pair's (frame output | global output), the tokens VGGT's heads read.
        Copies in and out run on the current stream; returns after the copy out."""
        dev = self.tokens.device
        C, P = self.cfg.dim, self.cfg.tokens_per_frame
        if not hasattr(self, "_img_dev") or self._img_dev.shape != images_host.shape:
            self._img_dev = torch.empty(images_host.shape, dtype=F16, device=dev)
            self._cat = torch.empty(self.S_local, P, 2 * C, dtype=F16, device=dev)
        self._img_dev.copy_(images_host, non_blocking=True)
        outs = self.forward(self._img_dev)
        fr, gl = outs[-1]
        self._cat[..., :C].copy_(fr.view(self.S_local, P, C))
        self._cat[..., C:].copy_(gl.view(self.S_local, P, C))
        if out_host is None:
            out_host = torch.empty(self._cat.shape, dtype=F16, pin_memory=True)
        out_host.copy_(self._cat, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return out_host
