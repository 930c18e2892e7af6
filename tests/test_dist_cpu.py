"""CPU, world_size 2 (gloo): the frame-sharded block pair equals the unsharded one.

Each rank owns S/2 contiguous frames.  The frame block runs on local frames
only; the global block writes local K/V rows into the rank's slice of the
global K/V buffer, all-gathers it in place with the same helpers the GPU
runner uses (``qvggt_b200.dist``), and attends its local queries against all
keys.  The math is the CPU oracle's; the test checks the decomposition, the
buffer layout, the collective and the special-token frame offsets.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import model as om, rope as orope
from qvggt_b200 import dist as qd

S, P, C, H = 4, 74, 128, 2        # small frames (5 special + 69 = 3 rows of a 23-wide grid)
GRID_W = 23


def _cfg_block(gen):
    return om.random_block(gen, dim=C, mlp=4 * C, kind="f16", ls=0.3)


def _block_sharded(x_local, blk, pos_local, kind, rank, world):
    """Oracle block over this rank's tokens; global attention via the gathered K/V."""
    T = x_local.shape[0]
    h = om.layernorm(x_local, blk["norm1_w"], blk["norm1_b"])
    qkv = blk["qkv"](h).reshape(T, 3, H, C // H)
    q = orope.rope2d(qkv[:, 0].permute(1, 0, 2), pos_local)            # [H, T, d]
    k = orope.rope2d(qkv[:, 1].permute(1, 0, 2), pos_local)
    v = qkv[:, 2].permute(1, 0, 2)
    if kind == "global":
        kv_local = torch.cat([k.permute(1, 0, 2).reshape(T, C), v.permute(1, 0, 2).reshape(T, C)], dim=1)
        kv_global = torch.empty(T * world, 2 * C, dtype=torch.float16)
        qd.kv_slice(kv_global, T, rank).copy_(kv_local)
        qd.gather_kv(kv_global, T, rank)
        kg = kv_global[:, :C].reshape(-1, H, C // H).permute(1, 0, 2)
        vg = kv_global[:, C:].reshape(-1, H, C // H).permute(1, 0, 2)
        o = om.sdpa(q, kg, vg)
    else:
        nf = T // P
        qf = q.reshape(H, nf, P, -1).permute(1, 0, 2, 3)
        kf = k.reshape(H, nf, P, -1).permute(1, 0, 2, 3)
        vf = v.reshape(H, nf, P, -1).permute(1, 0, 2, 3)
        o = om.sdpa(qf, kf, vf).permute(1, 0, 2, 3).reshape(H, T, -1)
    o = o.permute(1, 0, 2).reshape(T, C)
    x = om.r16(x_local.float() + om.r16(blk["proj"](o).float() * torch.as_tensor(blk["ls1"]).float()).float())
    h2 = om.layernorm(x, blk["norm2_w"], blk["norm2_b"])
    y = blk["fc2"](om.gelu_erf(blk["fc1"](h2)))
    return om.r16(x.float() + om.r16(y.float() * torch.as_tensor(blk["ls2"]).float()).float())


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = np.random.default_rng(0)
        fb, gb = _cfg_block(gen), _cfg_block(gen)
        tokens = torch.randn(S, P, C, generator=torch.Generator().manual_seed(1)).half()
        f0, nf = qd.frame_shard(S, world, rank)
        x = tokens[f0:f0 + nf].reshape(nf * P, C).clone()
        pos = orope.patch_positions(P, 5, GRID_W).repeat(nf, 1)
        x = _block_sharded(x, fb, pos, "frame", rank, world)
        x = _block_sharded(x, gb, pos, "global", rank, world)
        sets = [qd.special_token_set(f0 + i) for i in range(nf)]
        q.put((rank, x.numpy(), sets))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_frame_sharded_block_pair_equals_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, x, sets = q.get(timeout=300)
        res[r] = (x, sets)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    gen = np.random.default_rng(0)
    fb, gb = _cfg_block(gen), _cfg_block(gen)
    tokens = torch.randn(S, P, C, generator=torch.Generator().manual_seed(1)).half()
    _, ref = om.block_pair_forward(tokens, fb, gb, patch_start=5, grid_w=GRID_W)
    got = np.concatenate([res[r][0] for r in range(world)]).reshape(S, P, C)
    # CPU BLAS blocks the smaller per-rank matrices differently, so fp32 sums
    # differ in the last bits (a few fp16 ulps after rounding); a wrong shard,
    # offset or gather would be O(1).
    d = np.abs(got.astype(np.float32) - ref.numpy().astype(np.float32))
    assert d.max() <= 1e-2 and d.mean() <= 1e-3, (d.max(), d.mean())
    assert res[0][1] == [0, 1] and res[1][1] == [1, 1]


def test_frame_shard_rules():
    assert qd.frame_shard(32, 8, 3) == (12, 4)
    assert qd.frame_shard(200, 8, 7) == (175, 25)
    with pytest.raises(ValueError):
        qd.frame_shard(30, 8, 0)
    kv = torch.arange(12).reshape(6, 2)
    assert torch.equal(qd.kv_slice(kv, 2, 1), kv[2:4])


def _split_pass_worker(rank, world, port, q):
    """The GPU runner's split-pass global attention, restated with the oracle:
    local keys while the all-gather is in flight, then the other ranks' keys
    (``qvggt_b200.dist.remote_segments``), merged through the log-sum-exp."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        T, heads, d = 37, 2, 16
        g = torch.Generator().manual_seed(100 + rank)
        ql = torch.randn(heads, T, d, generator=g)
        kv_local = torch.randn(T, 2 * heads * d, generator=g).half()
        kv_global = torch.empty(T * world, 2 * heads * d, dtype=torch.float16)
        qd.kv_slice(kv_global, T, rank).copy_(kv_local)
        work = qd.gather_kv(kv_global, T, rank, async_op=True)

        def heads_of(rows):
            k = rows[:, :heads * d].reshape(-1, heads, d).permute(1, 0, 2)
            v = rows[:, heads * d:].reshape(-1, heads, d).permute(1, 0, 2)
            return k, v

        o1, l1 = om.sdpa_lse(ql, *heads_of(kv_local))          # overlaps the gather
        work.wait()
        segs = qd.remote_segments(T, world, rank)
        rem = torch.cat([kv_global[s:s + n] for s, n in segs])
        o2, l2 = om.sdpa_lse(ql, *heads_of(rem))
        o, lse = om.merge_attention([(o1, l1), (o2, l2)])
        ref_o, ref_lse = om.sdpa_lse(ql, *heads_of(kv_global))
        q.put((rank, float((o - ref_o).abs().max()), float((lse - ref_lse).abs().max()), segs))
    finally:
        dist.destroy_process_group()


def test_split_pass_global_attention_equals_full_world3():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 3
    port = _free_port()
    procs = [ctx.Process(target=_split_pass_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, eo, el, segs = q.get(timeout=300)
        res[r] = (eo, el, segs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r][0] <= 1e-5 and res[r][1] <= 1e-5, res[r]
    assert res[0][2] == [(37, 74)] and res[1][2] == [(0, 37), (74, 37)] and res[2][2] == [(0, 74)]
