"""GPU: the allocation-free split attention (``qvggt_attention_split_static``).

Some callers cannot let a library allocate device memory: a host runtime
without a device allocator, code running inside a memory pool's own callbacks,
or an integration that has already claimed every byte of the GPU.  For them the
split-KV attention has an entry point whose scratch is a fixed array inside the
library (64 MiB per GPU that loads it); it takes only the caller's inputs and
outputs.  This test calls it through the C ABI, twice in a row (the second call
finds the first call's data in the shared array), and compares each result
with ``qvggt_attention_ex`` given scratch the test allocated: the same kernel,
split count and merge order, within the attention tests' bounds (rel-L2
<= 4e-3, max-abs <= 1.5e-2 * max|O|).  It also checks the size limit.

Kept in its own file, named to be collected after every other test, and
written to pass alone in a fresh process too.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _static(q, kv, out, heads, batches, Lq, Lkv, splits):
    from qvggt_b200 import _lib
    C = heads * 64
    _lib.call("qvggt_attention_split_static", ctypes.c_void_p(q.data_ptr()), q.stride(0),
              ctypes.c_void_p(kv.data_ptr()), kv.stride(0), 0, C, ctypes.c_void_p(out.data_ptr()), out.stride(0),
              batches, Lq, Lkv, heads, splits, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _close(a, b):
    d = (a.float() - b.float())
    return (d.norm() / b.float().norm()).item() <= 4e-3 and d.abs().max().item() <= 1.5e-2 * b.float().abs().max().item()


@pytest.mark.parametrize("batches,Lq,Lkv,splits", [(1, 2048, 8192, 3), (4, 1374, 1374, 2)])
def test_static_scratch_attention_matches_caller_scratch(batches, Lq, Lkv, splits):
    from qvggt_b200 import awq_inference_engine as eng
    heads = 16
    g = torch.Generator(device=DEV).manual_seed(Lq + splits)
    q = torch.randn(batches * Lq, heads * 64, generator=g, device=DEV).half()
    kv = torch.randn(batches * Lkv, 2 * heads * 64, generator=g, device=DEV).half()
    nbytes = eng.attention_scratch_bytes(batches, Lq, heads, splits)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    ref = eng.attention_ex(q, kv, heads, batches, Lq, Lkv, splits=splits, scratch=scratch)
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        _static(q, kv, out, heads, batches, Lq, Lkv, splits)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert _close(out, ref)


def test_static_scratch_rejects_shapes_beyond_the_array():
    """4 splits of 16 heads x 43,968 queries need ~730 MB of scratch: refused
    with a message naming the limit, before anything is launched."""
    from qvggt_b200._lib import QvggtError
    heads, Lq = 16, 43968
    q = torch.zeros(Lq, heads * 64, dtype=torch.float16, device=DEV)
    kv = torch.zeros(Lq, 2 * heads * 64, dtype=torch.float16, device=DEV)
    out = torch.empty_like(q)
    with pytest.raises(QvggtError, match="fixed array"):
        _static(q, kv, out, heads, 1, Lq, Lq, 4)
