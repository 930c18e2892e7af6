"""Oracle: VGGT aggregator block math (CPU, PyTorch fp32 with fp16 rounding points).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

The aggregator itself lives in the un-vendored ``vggt-hf`` fork that the
reference imports (``qvggt/inference/loader.py:27``); its semantics are restated
here from the published VGGT algorithm and BASELINE config 1:

    x = x + ls1 * proj(attn(rope2d(q), rope2d(k), v)),  q,k,v = qkv(LN1(x))
    x = x + ls2 * fc2(gelu(fc1(LN2(x))))

pre-LayerNorm eps 1e-6, 16 heads x 64, LayerScale gamma, exact-erf GELU, 2-D
RoPE base 100, optional per-head q/k LayerNorm (``qk_norm``, off by default).
Every tensor that eager fp16 PyTorch would materialise is rounded to fp16 at
the same point; matmuls and reductions run in fp32.

The quantised linears follow ``WQLinear.forward`` (``qmodule.py:333-369``):
fp16 GEMM output, then a separate fp16 bias add.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import awq, rope

F16 = torch.float16


def r16(x: torch.Tensor) -> torch.Tensor:
    return x.to(F16)


def layernorm(x: torch.Tensor, w, b, eps: float = 1e-6) -> torch.Tensor:
    """fp16 in -> fp32 math -> fp16 out (as ``nn.LayerNorm`` on fp16)."""
    xf = x.float()
    mu = xf.mean(-1, keepdim=True)
    var = ((xf - mu) ** 2).mean(-1, keepdim=True)
    y = (xf - mu) * torch.rsqrt(var + eps)
    y = y * torch.as_tensor(w).float() + torch.as_tensor(b).float()
    return r16(y)


def gelu_erf(x: torch.Tensor) -> torch.Tensor:
    xf = x.float()
    return r16(0.5 * xf * (1.0 + torch.erf(xf / math.sqrt(2.0))))


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, chunk: int | None = None) -> torch.Tensor:
    """softmax(q k^T / sqrt(d)) v in fp32, q/k/v [..., L, d] fp16 -> fp16.
    Query rows are processed in chunks so the score block stays near 2e8 floats."""
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d)
    kf, vf = k.float(), v.float()
    if chunk is None:
        lead = max(1, q[..., 0, 0].numel())
        chunk = max(64, int(2e8 // (lead * k.shape[-2])))
    outs = []
    for s in range(0, q.shape[-2], chunk):
        qf = q[..., s:s + chunk, :].float()
        a = torch.softmax((qf @ kf.transpose(-1, -2)) * scale, dim=-1)
        outs.append(a @ vf)
    return r16(torch.cat(outs, dim=-2))


def sdpa_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """softmax(q k^T / sqrt(d)) v in fp32 and the natural log-sum-exp of each
    row's scaled scores; q/k/v [..., L, d].  Returns (o fp32, lse fp32 [..., Lq])."""
    d = q.shape[-1]
    s = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(d)
    lse = torch.logsumexp(s, dim=-1)
    return torch.exp(s - lse[..., None]) @ v.float(), lse


def merge_attention(parts) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact merge of attention results over disjoint key sets: parts is a list
    of (o, lse); o = sum_i exp(lse_i - lse) o_i with lse = logsumexp_i lse_i."""
    lses = torch.stack([p[1] for p in parts])
    lse = torch.logsumexp(lses, dim=0)
    o = sum(torch.exp(p[1] - lse)[..., None] * p[0].float() for p in parts)
    return o, lse


class QLinear:
    """One linear in the W4A16 (``kind='w4'``), dense fp16 (``'f16'``) or
    W8A8 (``'w8'``) form, holding exactly the buffers the GPU path uses."""

    def __init__(self, kind: str, **bufs):
        self.kind = kind
        self.__dict__.update(bufs)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """fp16 [.., K] -> fp16 [.., N] including the bias."""
        if self.kind == "w4":
            return awq.wqlinear_forward_fp16(x, self.qweight, self.scales, self.scaled_zeros,
                                             self.group_size, self.bias)
        if self.kind == "f16":
            y = r16(x.reshape(-1, x.shape[-1]).float() @ torch.as_tensor(self.weight).float().t())
            if self.bias is not None:
                y = r16(y.float() + torch.as_tensor(self.bias).float())
            return y.reshape(*x.shape[:-1], -1)
        raise ValueError(self.kind)

    def w8a8(self, xq, xs) -> torch.Tensor:
        """int8 activations [T, K] + per-token fp16 scales -> fp16 [T, N]
        (the reference's fused-bias W8A8 GEMM epilogue)."""
        from . import w8a8 as ow
        return torch.from_numpy(ow.w8a8_gemm(np.asarray(xq), np.asarray(self.w8), np.asarray(self.wscale),
                                             np.asarray(xs), None if self.bias is None else np.asarray(self.bias)))


def random_w4_linear(K: int, N: int, gen: np.random.Generator, group_size: int = 128,
                     w_std: float = 0.02) -> QLinear:
    """Random-init nn.Linear weights N(0, w_std), quantised W4A16 the AWQ way
    (asymmetric per group: s = (max-min)/15, z = round(-min/s))."""
    G = group_size
    w = gen.standard_normal((N, K)).astype(np.float32) * w_std
    wg = w.reshape(N, K // G, G)
    mx, mn = wg.max(-1), wg.min(-1)
    s = np.maximum((mx - mn) / 15.0, 1e-5).astype(np.float16)
    z = np.clip(np.round(-mn / s.astype(np.float32)), 0, 15).astype(np.float32)
    q = np.clip(np.round(wg / s.astype(np.float32)[..., None] + z[..., None]), 0, 15).astype(np.int32)
    q = q.reshape(N, K)
    gpad = awq.calculate_zeros_width(K, G) * 8
    st = np.zeros((gpad, N), np.float16)
    st[: K // G] = s.T
    szt = np.zeros((gpad, N), np.float16)
    szt[: K // G] = (-(s.astype(np.float32) * z)).astype(np.float16).T
    bias = (gen.standard_normal(N) * 0.01).astype(np.float16)
    return QLinear("w4", qweight=awq.pack_intweight(q), scales=st, scaled_zeros=szt, bias=bias,
                   group_size=G, in_features=K, out_features=N)


def random_f16_linear(K: int, N: int, gen: np.random.Generator, w_std: float = 0.02) -> QLinear:
    w = (gen.standard_normal((N, K)) * w_std).astype(np.float16)
    bias = (gen.standard_normal(N) * 0.01).astype(np.float16)
    return QLinear("f16", weight=w, bias=bias, in_features=K, out_features=N)


def random_block(gen: np.random.Generator, dim: int = 1024, mlp: int = 4096, kind: str = "w4",
                 ls: float = 0.01, qk_norm: bool = False, head_dim: int = 64) -> dict:
    mk = (lambda K, N: random_w4_linear(K, N, gen)) if kind == "w4" else (lambda K, N: random_f16_linear(K, N, gen))
    blk = dict(
        norm1_w=(1.0 + 0.1 * gen.standard_normal(dim)).astype(np.float16),
        norm1_b=(0.1 * gen.standard_normal(dim)).astype(np.float16),
        qkv=mk(dim, 3 * dim), proj=mk(dim, dim),
        ls1=np.full(dim, ls, np.float16),
        norm2_w=(1.0 + 0.1 * gen.standard_normal(dim)).astype(np.float16),
        norm2_b=(0.1 * gen.standard_normal(dim)).astype(np.float16),
        fc1=mk(dim, mlp), fc2=mk(mlp, dim),
        ls2=np.full(dim, ls, np.float16),
        qk_norm=qk_norm,
    )
    if qk_norm:
        blk.update(qn_w=(1.0 + 0.1 * gen.standard_normal(head_dim)).astype(np.float16),
                   qn_b=(0.1 * gen.standard_normal(head_dim)).astype(np.float16),
                   kn_w=(1.0 + 0.1 * gen.standard_normal(head_dim)).astype(np.float16),
                   kn_b=(0.1 * gen.standard_normal(head_dim)).astype(np.float16))
    return blk


def block_forward(x: torch.Tensor, blk: dict, pos: torch.Tensor | None, heads: int = 16,
                  eps: float = 1e-6, attn_fn=None) -> torch.Tensor:
    """One pre-LN transformer block over x [B, L, C] fp16 with positions pos [L, 2]
    (``None`` disables RoPE).  Returns fp16 [B, L, C]."""
    B, L, C = x.shape
    hd = C // heads
    h = layernorm(x, blk["norm1_w"], blk["norm1_b"], eps)
    qkv = blk["qkv"](h).reshape(B, L, 3, heads, hd).permute(2, 0, 3, 1, 4)
    q, k, v = qkv[0], qkv[1], qkv[2]
    if blk.get("qk_norm"):
        q = layernorm(q, blk["qn_w"], blk["qn_b"], eps)
        k = layernorm(k, blk["kn_w"], blk["kn_b"], eps)
    if pos is not None:
        q = rope.rope2d(q, pos)
        k = rope.rope2d(k, pos)
    o = (attn_fn or sdpa)(q, k, v)
    o = o.transpose(1, 2).reshape(B, L, C)
    y = blk["proj"](o)
    x = r16(x.float() + r16(y.float() * torch.as_tensor(blk["ls1"]).float()).float())
    h2 = layernorm(x, blk["norm2_w"], blk["norm2_b"], eps)
    f = gelu_erf(blk["fc1"](h2))
    y2 = blk["fc2"](f)
    return r16(x.float() + r16(y2.float() * torch.as_tensor(blk["ls2"]).float()).float())


def block_forward_w8a8(x: torch.Tensor, blk: dict, pos: torch.Tensor, heads: int = 16,
                       eps: float = 1e-6) -> torch.Tensor:
    """W8A8 block over x [B, L, C], the chain the
    reference's W8A8 kernels imply (``csrc/w8a8``): rms_norm_general ->
    int8 GEMM + bias -> 2-D RoPE -> attention -> invoke_quant -> int8 GEMM +
    bias -> LayerScale residual -> rms_norm_general -> int8 GEMM + bias ->
    gelu_and_quant (tanh GELU) -> int8 GEMM + bias -> LayerScale residual."""
    from . import w8a8 as ow
    B, L, C = x.shape
    hd = C // heads
    xf = x.reshape(B * L, C)
    q8, s = ow.rms_norm_general(xf.numpy(), np.asarray(blk["norm1_w"]), np.asarray(blk["norm1_b"]), eps)
    qkv = blk["qkv"].w8a8(q8, s).reshape(B, L, 3, heads, hd).permute(2, 0, 3, 1, 4)
    q = rope.rope2d(qkv[0], pos)
    k = rope.rope2d(qkv[1], pos)
    o = sdpa(q, k, qkv[2]).transpose(1, 2).reshape(B * L, C)
    oq, os_ = ow.invoke_quant(o.numpy())
    y = blk["proj"].w8a8(oq, os_)
    xf = r16(xf.float() + r16(y.float() * torch.as_tensor(blk["ls1"]).float()).float())
    q8, s = ow.rms_norm_general(xf.numpy(), np.asarray(blk["norm2_w"]), np.asarray(blk["norm2_b"]), eps)
    f = blk["fc1"].w8a8(q8, s)
    fq, fs, _ = ow.gelu_and_quant(f.numpy())
    y2 = blk["fc2"].w8a8(fq, fs)
    xf = r16(xf.float() + r16(y2.float() * torch.as_tensor(blk["ls2"]).float()).float())
    return xf.reshape(B, L, C)


def block_pair_forward(tokens: torch.Tensor, frame_blk: dict, global_blk: dict,
                       patch_start: int = 5, grid_w: int = 37) -> tuple[torch.Tensor, torch.Tensor]:
    """Frame block over [S, P, C] then global block over [1, S*P, C].

    Returns (frame_out [S, P, C], global_out [S, P, C]).
    """
    S, P, C = tokens.shape
    pos = rope.patch_positions(P, patch_start, grid_w)
    xf = block_forward(tokens, frame_blk, pos)
    xg = block_forward(xf.reshape(1, S * P, C), global_blk, pos.repeat(S, 1))
    return xf, xg.reshape(S, P, C)


# --------------------------------------------------------------- DINOv2 front
# The aggregator's patch embed is a DINOv2 ViT-L/14 with 4 register tokens,
# kept in fp16 and unquantised (the reference excludes it from quantisation at
# ``qvggt/inference/loader.py:346``).  Its forward, restated from the published
# DINOv2 / VGGT models (vggt-hf is not vendored, so this is unpinned):
#   images in [0, 1] -> (x - mean) / std (ImageNet statistics, fp16 ops)
#   -> 14x14 stride-14 convolution (+ bias) = patch tokens
#   -> [cls + pos[0] | 4 registers | patches + pos[1:]]
#   -> 24 pre-LN blocks without RoPE (LayerScale, exact-erf GELU)
#   -> final LayerNorm; the patch rows are the aggregator's patch tokens.

IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def patchify(images: torch.Tensor, patch: int = 14, mean=IMAGENET_MEAN, std=IMAGENET_STD) -> torch.Tensor:
    """images fp16 [S, 3, H, W] -> normalised patches fp16 [S * (H/p) * (W/p), 3*p*p],
    column c*p*p + ky*p + kx (the flattened conv weight's order).  The
    normalisation rounds to fp16 after the subtraction and after the division
    (an fp16 model's buffers and arithmetic)."""
    S, Cin, H, W = images.shape
    m = torch.tensor(mean, dtype=F16).float().view(1, 3, 1, 1)
    s = torch.tensor(std, dtype=F16).float().view(1, 3, 1, 1)
    x = r16(r16(images.float() - m).float() / s)
    x = x.reshape(S, Cin, H // patch, patch, W // patch, patch).permute(0, 2, 4, 1, 3, 5)
    return x.reshape(S * (H // patch) * (W // patch), Cin * patch * patch).contiguous()


def patch_embed_forward(images: torch.Tensor, pe: dict, heads: int = 16, eps: float = 1e-6) -> torch.Tensor:
    """DINOv2 front over images [S, 3, H, W] fp16 -> normalised tokens fp16
    [S, 5 + n_patch, C] ([cls | 4 registers | patches] after the final LayerNorm).

    ``pe`` holds: ``patch_w`` [C, 3*p*p] fp16, ``patch_b`` [C], ``cls`` [C],
    ``registers`` [4, C], ``pos_cls`` [C], ``pos_patch`` [n_patch, C],
    ``blocks`` (dicts for :func:`block_forward`, dense fp16 linears),
    ``norm_w`` / ``norm_b``, ``patch``."""
    S = images.shape[0]
    p = pe["patch"]
    x = patchify(images, p)
    n = x.shape[0] // S
    C = pe["patch_w"].shape[0]
    lin = QLinear("f16", weight=pe["patch_w"], bias=pe["patch_b"])
    tok = lin(x).reshape(S, n, C)
    pos_p = torch.as_tensor(pe["pos_patch"]).float()
    pos_c = torch.as_tensor(pe["pos_cls"]).float()
    cls = r16(torch.as_tensor(pe["cls"]).float() + pos_c).reshape(1, 1, C).expand(S, 1, C)
    regs = torch.as_tensor(pe["registers"]).to(F16).reshape(1, -1, C).expand(S, -1, C)
    patches = r16(tok.float() + pos_p)
    x = torch.cat([cls, regs, patches], dim=1).contiguous()
    for blk in pe["blocks"]:
        x = block_forward(x, blk, None, heads, eps)
    return layernorm(x, pe["norm_w"], pe["norm_b"], eps)


def aggregator_tokens(pe_out: torch.Tensor, specials: torch.Tensor, frame_offset: int = 0,
                      patch_start: int = 5) -> torch.Tensor:
    """[S, 5 + n, C] DINOv2 output -> aggregator input [S, 5 + n, C]: the
    DINOv2 special rows are dropped and replaced by the aggregator's camera +
    register tokens, set 0 for the first frame of the sequence (global frame
    index 0) and set 1 for every other frame.  ``specials`` is [2, 5, C]."""
    S = pe_out.shape[0]
    sp = torch.as_tensor(specials).to(F16)
    rows = [sp[0 if (f + frame_offset) == 0 else 1] for f in range(S)]
    return torch.cat([torch.stack(rows), pe_out[:, patch_start:]], dim=1).contiguous()


def aggregator_forward(images: torch.Tensor, pe: dict, specials, frame_blocks: list, global_blocks: list,
                       patch_start: int = 5):
    """The full aggregator on S frames: DINOv2 front, special tokens, then the
    frame / global block pairs (2-D RoPE over the frames' patch grid, its width
    = image width / patch).  Returns (aggregator input tokens, last frame block
    output, last global block output), each [S, P, C]."""
    x = aggregator_tokens(patch_embed_forward(images, pe), specials, 0, patch_start)
    grid_w = images.shape[-1] // pe["patch"]
    x0 = x
    xf = x
    for fb, gb in zip(frame_blocks, global_blocks):
        xf, x = block_pair_forward(x, fb, gb, patch_start, grid_w)
    return x0, xf, x


# ------------------------------------------------------- other frame sizes
def _aa_bicubic_weights(n_in: int, n_out: int, a: float = -0.5) -> np.ndarray:
    """[n_out, n_in] resampling matrix of separable antialiased bicubic
    interpolation: output sample i sits at input coordinate (i + 0.5) * scale,
    scale = n_in / n_out; the Keys cubic (a = -0.5) is stretched by
    max(scale, 1) when shrinking, taps are cut to the image and each row is
    normalised to sum 1 (the published separable-resampling method, as in
    Pillow's and PyTorch's antialiased resize)."""
    def cubic(x):
        x = abs(x)
        if x < 1.0:
            return (a + 2.0) * x ** 3 - (a + 3.0) * x ** 2 + 1.0
        if x < 2.0:
            return a * x ** 3 - 5.0 * a * x ** 2 + 8.0 * a * x - 4.0 * a
        return 0.0
    scale = n_in / n_out
    fs = max(scale, 1.0)
    support = 2.0 * fs
    W = np.zeros((n_out, n_in), np.float64)
    for i in range(n_out):
        center = (i + 0.5) * scale
        lo = max(int(center - support + 0.5), 0)
        hi = min(int(center + support + 0.5), n_in)
        w = np.array([cubic((x - center + 0.5) / fs) for x in range(lo, hi)])
        W[i, lo:hi] = w / w.sum()
    return W


def interpolate_pos_embed(pos_embed, rows: int, cols: int) -> torch.Tensor:
    """DINOv2's position table [1 + M*M, C] resampled to a rows x cols patch
    grid (class position kept; patch grid resized as an image, bicubic with
    antialiasing, in float64 here).  Returns fp32 [1 + rows*cols, C]."""
    pe = np.asarray(torch.as_tensor(pos_embed).float(), np.float64)
    M = int(round(math.sqrt(pe.shape[0] - 1)))
    grid = pe[1:].reshape(M, M, -1)
    out = np.einsum("ri,ijc,sj->rsc", _aa_bicubic_weights(M, rows), grid, _aa_bicubic_weights(M, cols))
    return torch.from_numpy(np.concatenate([pe[:1], out.reshape(rows * cols, -1)]).astype(np.float32))
