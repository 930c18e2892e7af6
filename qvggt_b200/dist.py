"""Frame sharding across ranks (one process per GPU).

Frames are split into equal contiguous shards; everything but the global
blocks' attention is rank-local.  A global block needs every frame's K/V: each
rank writes its own rows into its slice of a [S*P, 2C] buffer and the buffer
is all-gathered in place (NCCL over NVLink / NVSwitch on GPUs; the same call
works with gloo on CPU ranks, which is how the tests exercise it).  These
helpers hold the layout decisions so that the runner and the CPU tests share
them.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def frame_shard(S: int, world: int, rank: int) -> tuple[int, int]:
    """(first global frame, number of frames) owned by ``rank``."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    if S % world:
        raise ValueError(f"{S} frames do not split evenly over {world} ranks")
    n = S // world
    return rank * n, n


def kv_slice(kv_global: torch.Tensor, rows_local: int, rank: int) -> torch.Tensor:
    """This rank's rows of the global K/V buffer (where its qkv epilogue writes)."""
    return kv_global[rank * rows_local:(rank + 1) * rows_local]


def gather_kv(kv_global: torch.Tensor, rows_local: int, rank: int, group=None, async_op: bool = False):
    """All-gather every rank's K/V rows into ``kv_global`` in place.  Returns
    ``kv_global``, or with ``async_op`` the collective's work handle (its
    ``wait()`` makes the current stream wait for the gather)."""
    work = dist.all_gather_into_tensor(kv_global, kv_slice(kv_global, rows_local, rank), group=group,
                                       async_op=async_op)
    return work if async_op else kv_global


def remote_segments(rows_local: int, world: int, rank: int) -> list[tuple[int, int]]:
    """The other ranks' rows of the gathered K/V buffer as (start, length)
    ranges: the rows before this rank's slice and the rows after it (empty
    ranges dropped).  A rank attends to its own slice while the all-gather is
    in flight, then to these rows."""
    before = (0, rank * rows_local)
    after = ((rank + 1) * rows_local, (world - 1 - rank) * rows_local)
    return [sg for sg in (before, after) if sg[1] > 0]


def special_token_set(global_frame: int) -> int:
    """VGGT gives the first frame of the sequence its own camera / register
    tokens (set 0) and every other frame set 1."""
    return 0 if global_frame == 0 else 1
