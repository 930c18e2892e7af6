"""GPU, 2 and 4 ranks (NCCL): the frame-sharded aggregator equals the single-GPU one.

Runs as child processes, one per GPU, when enough GPUs are visible (skipped
otherwise).  Rank r owns frames [r*S/N, (r+1)*S/N); global blocks all-gather
K/V over NCCL while the rank attends to its own keys, then attend to the other
ranks' keys and merge the two passes (at 4 ranks the middle ranks' remote keys
are two segments).  Rank 0 also runs the whole sequence alone on its GPU and
compares: rel-L2 <= 2e-3 (the split passes round each part to fp16 before the
merge).  NVLS is switched off (NCCL_NVLS_ENABLE=0) and no kernel reads peer
memory.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import os, sys, datetime, torch, torch.distributed as dist
sys.path.insert(0, os.environ["QV_ROOT"])
from qvggt_b200 import _lib
from qvggt_b200.aggregator import AggConfig
from qvggt_b200.synthetic import random_vggt_aggregator, synthetic_images
from qvggt_b200.dist import frame_shard
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
_lib.load()
S = 8
cfg = AggConfig(depth=2)
f0, n = frame_shard(S, world, rank)
m = random_vggt_aggregator(cfg, 7, torch.device("cuda", rank), n, dist.group.WORLD, world, rank, pe_depth=2)
imgs = synthetic_images(S, 3)
outs = m.forward(imgs[f0:f0 + n].contiguous().cuda())
fr, gl = outs[-1]
gathered = [torch.empty_like(gl) for _ in range(world)]
dist.all_gather(gathered, gl.contiguous())
torch.cuda.synchronize()
if rank == 0:
    full = torch.cat(gathered).float().cpu()
    single = random_vggt_aggregator(cfg, 7, torch.device("cuda", 0), S, None, 1, 0, pe_depth=2)
    ref = single.forward(imgs.cuda())[-1][1].float().cpu()
    err = ((full - ref).norm() / ref.norm()).item()
    print("REL_L2", err, flush=True)
    assert err <= 2e-3, err
    assert _lib.device_status() == 0
dist.barrier()
dist.destroy_process_group()
"""


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 4])
def test_frame_sharded_aggregator_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), QV_ROOT=ROOT, NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, "-c", WORKER], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=600)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append(out)
    assert all(p.returncode == 0 for p in procs), "\n".join(o[-2000:] for o in outs)
    assert "REL_L2" in outs[0]
