"""Small, fixed workloads of single kernels for profiling (ncu) and timing.

    python profile_cases.py attn  [L] [batches]   # flash attention, 16 heads x 64
    python profile_cases.py gemm  f16|w4|w8 [M]    # tcgen05 GEMM, N=4096 K=1024
    python profile_cases.py mem                    # LayerNorm, invoke_quant, GEMV
    python profile_cases.py small [M] [N] [K]      # small-M split-K GEMM (camera trunk)
    python profile_cases.py small_time             # small-M vs large kernel vs GEMV
    python profile_cases.py trunk                  # camera-head trunk (4 blocks, width 2048)
    python profile_cases.py forward w4|w8 [S] [n]  # whole aggregator forward, frames/s
    python profile_cases.py time                   # CUDA-event timings of all of the above
    python profile_cases.py sdpa                   # torch SDPA backends vs ours at the bench's attention shapes
    python profile_cases.py ranks [S]              # global attention of one rank of N = 1, 2, 4, 8 (split plans)
    python profile_cases.py gemm_configs           # every GEMM kernel configuration at per-rank shapes
    python profile_cases.py gemv [N] [K] [m]       # the W4A16 GEMV alone (two launches, one weight set)

Each case launches its kernel twice (so `ncu -s 1 -c 1` captures a warm
launch) on seeded synthetic data sized above the 126 MB L2 where it matters.
"""
from __future__ import annotations

import sys

import torch

import os

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from qvggt_b200 import _lib  # noqa: E402
from qvggt_b200 import awq_inference_engine as eng  # noqa: E402


def _w4(N, K, seed=1):
    from qvggt_b200.synthetic import quantize_w4
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(N, K, generator=g, device="cuda") * 0.02
    return quantize_w4(w, 128)


def attn(L=16384, b=1, reps=2):
    C = 1024
    q = torch.randn(b * L, C, dtype=torch.float16, device="cuda")
    kv = torch.randn(b * L, 2 * C, dtype=torch.float16, device="cuda")
    out = torch.empty(b * L, C, dtype=torch.float16, device="cuda")
    fn = lambda: eng.attention(q, kv, 16, b, L, L, out=out)
    for _ in range(reps):
        fn()
    return fn, 4.0 * b * L * L * C


def gemm(mode="f16", M=32768, N=4096, K=1024, reps=2):
    x = torch.randn(M, K, dtype=torch.float16, device="cuda")
    if mode == "f16":
        w = torch.randn(N, K, dtype=torch.float16, device="cuda") * 0.02
        out = torch.empty(M, N, dtype=torch.float16, device="cuda")
        fn = lambda: eng.f16_linear(x, w, out=out)
    elif mode == "w4":
        qw, s, z = _w4(N, K)
        fn = lambda: eng.gemm_forward_cuda_new(x, qw, s, z)
    else:
        a8 = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
        w8 = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda")
        ws = torch.rand(N, device="cuda").half() * 1e-3
        as_ = torch.rand(M, device="cuda").half() * 1e-2
        out = torch.empty(M, N, dtype=torch.float16, device="cuda")
        fn = lambda: eng.w8a8_gemm_forward_cuda(a8, w8, ws, as_, out)
    for _ in range(reps):
        fn()
    return fn, 2.0 * M * N * K


def mem(reps=2):
    T = 43968
    x = torch.randn(T, 1024, dtype=torch.float16, device="cuda")
    w1 = torch.ones(1024, dtype=torch.float16, device="cuda")
    q8 = torch.empty(T, 1024, dtype=torch.int8, device="cuda")
    sc = torch.empty(T, dtype=torch.float16, device="cuda")
    qw, s, z = _w4(4096, 4096)
    x1 = torch.randn(1, 4096, dtype=torch.float16, device="cuda")
    fns = {
        "layernorm [43968,1024]": (lambda: eng.layernorm(x, w1, w1), 2 * T * 1024 * 2),
        "invoke_quant [43968,1024]": (lambda: eng.invoke_quant(q8, x, sc), T * 1024 * 3 + 2 * T),
        "gemv m=1 N=K=4096": (lambda: eng.gemv_forward_cuda_new(x1, qw, s, z, 1, 4096, 4096, 128),
                              4096 * 4096 // 2 + 2 * s.numel() * 2 + 4096 * 4),
    }
    for f, _ in fns.values():
        for _ in range(reps):
            f()
    return fns


def gemv(N=4096, K=4096, m=1, reps=2):
    """The GEMV on one weight set, launched `reps` times (ncu -s 1 -c 1
    captures a warm-launch of the same kernel; ncu flushes the caches before
    each replay, so its DRAM figures are those of a cold read of the weights)."""
    qw, s, z = _w4(N, K)
    x = torch.randn(m, K, dtype=torch.float16, device="cuda")
    fn = lambda: eng.gemv_forward_cuda_new(x, qw, s, z, m, N, K, 128)
    for _ in range(reps):
        fn()
    nbytes = N * K // 2 + 2 * (K // 128) * N * 2 + m * K * 2 + m * N * 2
    return fn, nbytes


def small(M=32, N=6144, K=2048, reps=2):
    qw, s, z = _w4(N, K)
    x = torch.randn(M, K, dtype=torch.float16, device="cuda")
    out = torch.empty(M, N, dtype=torch.float16, device="cuda")
    fn = lambda: eng.small_linear(x, qw, s, z, out=out)
    for _ in range(reps):
        fn()
    return fn


def _rotating(N, K, total=256 << 20):
    """Enough copies of a W4 weight that cycling through them streams > L2."""
    wbytes = N * K // 2 + 2 * (K // 128) * N * 2
    return [_w4(N, K, seed=i) for i in range(max(2, -(-total // wbytes)))]


def small_time():
    """Camera-trunk linears (dim 2048) at M = 1..256 rows: the split-K small-M
    kernel, the large tcgen05 kernel and (M <= 16) the GEMV, each cycling
    through weight copies larger than L2 (HBM-bound), CUDA-graph replay."""
    for N, K in ((6144, 2048), (2048, 2048), (8192, 2048), (2048, 8192)):
        ws = _rotating(N, K)
        wbytes = N * K // 2 + 2 * (K // 128) * N * 2
        for M in (1, 8, 16, 32, 64, 128, 192, 256):
            x = torch.randn(M, K, dtype=torch.float16, device="cuda")
            out = torch.empty(M, N, dtype=torch.float16, device="cuda")
            nbytes = wbytes + M * K * 2 + M * N * 2
            it = [0]

            def nxt():
                w = ws[it[0] % len(ws)]
                it[0] += 1
                return w

            def f_small():
                qw, s, z = nxt()
                eng.small_linear(x, qw, s, z, out=out)

            def f_large():
                qw, s, z = nxt()
                _lib.call("qvggt_w4a16_linear_ex", x.data_ptr(), K, qw.data_ptr(), s.data_ptr(), z.data_ptr(), None,
                          out.data_ptr(), N, M, N, K, s.shape[0], 128, 0, None, 0, None,
                          torch.cuda.current_stream().cuda_stream)

            def f_gemv():
                qw, s, z = nxt()
                eng.gemv_forward_cuda_new(x, qw, s, z, M, N, K, 128)

            pl = eng.small_linear_plan(0, M, N, K)
            row = [f"N={N} K={K} M={M} [splits {pl['splits']} ctas {pl['ctas']} active {pl['active_clusters']}]:"]
            cases = [("small", f_small), ("large", f_large)] + ([("gemv", f_gemv)] if M <= 16 else [])
            for name, f in cases:
                t = _time(f, len(ws), graph=True)
                row.append(f"{name} {t * 1e6:.2f} us ({nbytes / t / 1e9:.0f} GB/s)")
            print("  ".join(row))


def trunk_time():
    """Camera-head trunk forward (4 W4A16 blocks of width 2048) over S camera
    tokens, CUDA-graph replay; the per-block algorithmic work is
    2 * S * 2048 * (6144 + 2048 + 8192 + 8192) + 4 * S^2 * 2048 FLOP."""
    from qvggt_b200.camera_trunk import random_camera_trunk
    trunk = random_camera_trunk(seed=1, device="cuda", depth=4)
    for S in (8, 32, 64, 200):
        x = torch.randn(1, S, 2048, device="cuda").half()
        t = _time(lambda: trunk(x), 20, graph=True)
        fl = 4 * (2 * S * 2048 * (6144 + 2048 + 8192 + 8192) + 4 * S * S * 2048)
        wbytes = 4 * 2048 * (6144 + 2048 + 8192 + 8192) // 2
        print(f"camera trunk S={S}: {t * 1e6:.1f} us ({fl / t / 1e12:.2f} TFLOP/s, W4 weights {wbytes / t / 1e9:.0f} GB/s)")


def forward_time(kind="w4", S=32, steps=3):
    """Frames/s of the full aggregator forward (DINOv2 front + 24 pairs) on one
    GPU, images resident: kind "w4" is BASELINE config 2, "w8" (S = 64) the
    W8A8 aggregator of config 3."""
    from qvggt_b200.aggregator import AggConfig
    from qvggt_b200.synthetic import random_vggt_aggregator, synthetic_images
    agg = random_vggt_aggregator(AggConfig(), 0, "cuda", S, kind=kind)
    imgs = synthetic_images(S, 0).cuda()
    agg.forward(imgs)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    for _ in range(steps):
        agg.forward(imgs)
    b.record()
    torch.cuda.synchronize()
    t = a.elapsed_time(b) / steps / 1e3
    print(f"aggregator forward {kind} S={S}: {t * 1e3:.1f} ms, {S / t:.2f} frames/s")


def sdpa_bar(iters=5):
    """torch's scaled_dot_product_attention (each fp16 backend this build
    offers: cuDNN, flash, memory-efficient) against this library's kernel at
    the benchmark's attention shapes: the global block at S = 32 on one GPU
    (1 x 16 heads x 43,968 tokens), the frame blocks (32 x 16 x 1,374) and the
    global block of 8-GPU ranks (Lq = 5,496 against 43,968).  CUDA events,
    warm launches; SM clocks sampled during the timed loops."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    from bench import ClockSampler
    shapes = [("global S=32", 1, 43968, 43968), ("frame S=32", 32, 1374, 1374), ("global rank of 8", 1, 5496, 43968)]
    backends = [("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION),
                ("efficient", SDPBackend.EFFICIENT_ATTENTION)]
    with ClockSampler(torch.cuda.current_device()) as clk:
        for name, b, Lq, Lkv in shapes:
            C = 1024
            q = torch.randn(b * Lq, C, dtype=torch.float16, device="cuda")
            kv = torch.randn(b * Lkv, 2 * C, dtype=torch.float16, device="cuda")
            out = torch.empty(b * Lq, C, dtype=torch.float16, device="cuda")
            fl = 4.0 * b * Lq * Lkv * C
            fn = lambda: eng.attention(q, kv, 16, b, Lq, Lkv, out=out)
            fn()
            t = _time(fn, iters)
            row = [f"{name} (b={b}, Lq={Lq}, Lkv={Lkv}): qvggt {t * 1e3:.3f} ms {fl / t / 1e12:.0f} TFLOP/s"]
            qh = q.view(b, Lq, 16, 64).transpose(1, 2)
            kh = kv[:, :C].view(b, Lkv, 16, 64).transpose(1, 2)
            vh = kv[:, C:].view(b, Lkv, 16, 64).transpose(1, 2)
            for bname, be in backends:
                try:
                    with sdpa_kernel([be]):
                        f2 = lambda: F.scaled_dot_product_attention(qh, kh, vh)
                        f2()
                        t2 = _time(f2, iters)
                    row.append(f"sdpa-{bname} {t2 * 1e3:.3f} ms {fl / t2 / 1e12:.0f} TFLOP/s")
                except RuntimeError as e:
                    row.append(f"sdpa-{bname} unavailable ({str(e).splitlines()[0][:60]})")
            print("  ".join(row), flush=True)
    print("clocks during the timed loops:", clk.summary())


def rank_shapes(S=32, iters=5):
    """Global attention of one rank when S frames are sharded over N GPUs
    (Lq = S/N frames of queries against all S frames of keys): one launch
    over all keys, the same with the library's split plan, and the two-pass
    form the aggregator uses with N > 1 (own keys with lse, then the others'
    keys merged); TFLOP/s of the whole call."""
    from qvggt_b200.dist import remote_segments
    P, C, heads = 1374, 1024, 16
    Lkv = S * P
    kv = torch.randn(Lkv, 2 * C, dtype=torch.float16, device="cuda")
    for N in (1, 2, 4, 8):
        if S % N:
            continue
        T = S // N * P
        q = torch.randn(T, C, dtype=torch.float16, device="cuda")
        out = torch.empty(T, C, dtype=torch.float16, device="cuda")
        lse = torch.empty(heads, T, dtype=torch.float32, device="cuda")
        fl = 4.0 * T * Lkv * C
        sp_all, nb_all = eng.attention_plan(1, T, Lkv, heads)
        sp_loc, nb1 = eng.attention_plan(1, T, T, heads)
        sp_rem, nb2 = eng.attention_plan(1, T, Lkv - T, heads) if N > 1 else (1, 0)
        scratch = torch.empty(max(nb_all, nb1, nb2, 256), dtype=torch.uint8, device="cuda")
        r = N // 2                                   # a middle rank: its remote keys are two segments at N >= 4

        def two_pass():
            eng.attention_ex(q, kv, heads, 1, T, Lkv, out=out, segments=[(r * T, T)], splits=sp_loc, lse=lse,
                             lse_mode=1, scratch=scratch)
            if N > 1:
                eng.attention_ex(q, kv, heads, 1, T, Lkv, out=out, segments=remote_segments(T, N, r), splits=sp_rem,
                                 lse=lse, lse_mode=2, scratch=scratch)

        cases = [("one launch", lambda: eng.attention(q, kv, heads, 1, T, Lkv, out=out)),
                 (f"split plan {sp_all}", lambda: eng.attention_ex(q, kv, heads, 1, T, Lkv, out=out, splits=sp_all,
                                                                  scratch=scratch)),
                 (f"local {sp_loc} + remote {sp_rem}", two_pass)]
        row = [f"N={N} (Lq={T}, Lkv={Lkv}):"]
        for name, f in cases:
            f()
            t = _time(f, iters)
            row.append(f"{name} {t * 1e3:.3f} ms {fl / t / 1e12:.0f} TFLOP/s")
        print("  ".join(row), flush=True)


def gemm_configs(iters=10):
    """The aggregator's linears at the per-rank row counts of 1, 2, 4 and 8
    GPUs (S = 32) under each kernel configuration (1 = CTA pairs, 2 = 1-SM
    256-wide, 3 = 1-SM 128-wide) and the automatic choice (0); W4A16 and
    dense fp16 (the DINOv2 front), TFLOP/s."""
    shapes = [(3072, 1024), (1024, 1024), (4096, 1024), (1024, 4096)]     # qkv, proj, fc1, fc2
    for M in (43968, 21984, 10992, 5496):
        for mode in ("w4", "f16"):
            for N, K in shapes:
                x = torch.randn(M, K, dtype=torch.float16, device="cuda")
                out = torch.empty(M, N, dtype=torch.float16, device="cuda")
                if mode == "w4":
                    qw, s, z = _w4(N, K)
                    fn = lambda: eng.w4a16_linear(x, qw, s, z, out=out)
                else:
                    w = torch.randn(N, K, dtype=torch.float16, device="cuda") * 0.02
                    fn = lambda: eng.f16_linear(x, w, out=out)
                row = [f"{mode} M={M} N={N} K={K}:"]
                for cfg in (0, 1, 2, 3):
                    _lib.call("qvggt_set_gemm_config", cfg)
                    fn()
                    t = _time(fn, iters)
                    row.append(f"cfg{cfg} {t * 1e6:.1f} us {2.0 * M * N * K / t / 1e12:.0f}")
                _lib.call("qvggt_set_gemm_config", 0)
                print("  ".join(row), flush=True)


def _time(fn, iters=20, graph=False):
    """Average device time per call.  graph=True captures the `iters` calls in
    one CUDA graph first, so host launch overhead does not pace short kernels."""
    torch.cuda.synchronize()
    if graph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        run = g.replay
    else:
        def run():
            for _ in range(iters):
                fn()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    run()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters / 1e3


def main(argv):
    _lib.load()
    what = argv[0] if argv else "time"
    if what == "attn":
        attn(*(int(v) for v in argv[1:3]))
    elif what == "gemm":
        gemm(argv[1] if len(argv) > 1 else "f16", *(int(v) for v in argv[2:3]))
    elif what == "mem":
        mem()
    elif what == "gemv":
        gemv(*(int(v) for v in argv[1:4]))
    elif what == "small":
        small(*(int(v) for v in argv[1:4]))
    elif what == "small_time":
        small_time()
    elif what == "trunk":
        trunk_time()
    elif what == "forward":
        forward_time(argv[1] if len(argv) > 1 else "w4", *(int(v) for v in argv[2:4]))
    elif what == "sdpa":
        sdpa_bar()
    elif what == "gemm_configs":
        gemm_configs()
    elif what == "ranks":
        rank_shapes(*(int(v) for v in argv[1:2]))
    elif what == "time":
        for L, b in ((16384, 1), (43968, 1), (1374, 32)):
            fn, fl = attn(L, b)
            t = _time(fn, 5)
            print(f"attention L={L} b={b}: {t * 1e3:.3f} ms {fl / t / 1e12:.0f} TFLOP/s")
        for mode in ("f16", "w4", "w8"):
            fn, fl = gemm(mode, 43968)
            t = _time(fn)
            print(f"gemm {mode} M=43968 N=4096 K=1024: {t * 1e6:.1f} us {fl / t / 1e12:.0f} T(FL)OP/s")
        for name, (fn, nbytes) in mem().items():
            t = _time(fn, 100, graph=True)
            print(f"{name}: {t * 1e6:.2f} us {nbytes / t / 1e9:.0f} GB/s (CUDA-graph replay)")
        # the BASELINE config 0 GEMV (M = 1, K = 1024, N = 4096)
        qw, s, z = _w4(4096, 1024)
        x1 = torch.randn(1, 1024, dtype=torch.float16, device="cuda")
        t = _time(lambda: eng.gemv_forward_cuda_new(x1, qw, s, z, 1, 4096, 1024, 128), 200, graph=True)
        print(f"gemv m=1 N=4096 K=1024: {t * 1e6:.2f} us {2246656 / t / 1e9:.0f} GB/s (CUDA-graph replay)")
    torch.cuda.synchronize()
    print("ok", what)


if __name__ == "__main__":
    main(sys.argv[1:])
