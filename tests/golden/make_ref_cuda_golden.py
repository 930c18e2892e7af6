"""Golden outputs of the reference's own CUDA kernels, run on a B200.

    python oracle/build_ref.py            # in the container with the reference checkout
    python tests/golden/make_ref_cuda_golden.py --out ref_cuda_golden.npz [--time]
    python tests/golden/make_ref_cuda_golden.py --gemm-pins ref_cuda_gemm_pins.npz
    python tests/golden/make_ref_cuda_golden.py --bf16-pins ref_cuda_bf16_pins.npz

Runs the reference kernels (built from their own sources into oracle/_ref/ by
oracle/build_ref.py) on inputs generated from fixed seeds (regenerated
identically by the tests, see ``cases()``), and stores only the outputs.
``--time`` also prints CUDA-event timings of the reference kernels at the
benchmark shapes.

Not run: the reference GEMM with M <= 32.  That path (gemm_w4a16_T1 with
SPLITK = 2) waits on split-K semaphores allocated with torch::empty, i.e.
uninitialised (gemm_cuda.cu:28, semaphore.h:35-43), and can spin forever.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


def cases():
    """Seeded inputs shared by this generator and the tests (numpy, CPU)."""
    from oracle import awq
    c = {}
    for name, (M, N, K, seed) in {"gemm_a": (300, 512, 1024, 10), "gemm_b": (256, 256, 4096, 11)}.items():
        lin = awq.make_quantized_linear(N, K, 128, seed=seed, bias=False)
        x = np.random.default_rng(seed + 100).standard_normal((M, K)).astype(np.float16)
        c[name] = dict(x=x, qweight=lin["qweight"], scales=lin["scales"], scaled_zeros=lin["scaled_zeros"])
    rng = np.random.default_rng(20)
    c["w8a8"] = dict(a=rng.integers(-127, 128, (200, 512)).astype(np.int8),
                     w=rng.integers(-127, 128, (256, 512)).astype(np.int8),
                     ws=(rng.random(256) * 1e-3 + 1e-4).astype(np.float16),
                     as_=(rng.random(200) * 1e-2 + 1e-3).astype(np.float16),
                     bias=(rng.standard_normal(256) * 0.1).astype(np.float16))
    rng = np.random.default_rng(21)
    c["quant"] = dict(x=(rng.standard_normal((200, 1024)) * 3).astype(np.float16))
    rng = np.random.default_rng(22)
    c["ln"] = dict(x=(rng.standard_normal((200, 1024)) * 2 + 0.5).astype(np.float16),
                   w=(1 + 0.1 * rng.standard_normal(1024)).astype(np.float16),
                   b=(0.1 * rng.standard_normal(1024)).astype(np.float16))
    rng = np.random.default_rng(23)
    c["gelu"] = dict(x=(rng.standard_normal((128, 1024)) * 2).astype(np.float16))
    rng = np.random.default_rng(24)
    c["rope"] = dict(x=rng.standard_normal((37, 2, 16, 64)).astype(np.float16),
                     freqs=(rng.random((2, 37, 32)) * 10).astype(np.float32))
    return c


# Rows of the config-0 output kept in the pin fixture: the first full tile and
# the ragged last one (1374 = 10 x 128 + 94).  A row of C depends only on its
# own row of A, so the GPU test computes the whole product and compares these.
C0_ROWS = list(range(0, 64)) + list(range(1310, 1374))


def gemm_pin_cases():
    """Inputs of the GEMM pins (numpy, CPU), regenerated identically by the tests.

    ``eye``: A = I (M = K = 1024, N = 512), so C = deq(W)^T: every output
    element is one dequantised weight (times 1, plus exact zeros), and the
    reference kernel's fp16 accumulation is exact -- the fixture is the
    reference's dequantised matrix bit for bit.  The per-group scales span
    2^-6 .. 2^6 times the config-0 distribution so the fp16 rounding of
    q*s + (-s*z) is exercised at every magnitude; all 16 nibble values and all
    16 zero points occur.  M = 1024 takes the reference's ``gemm_w4a16_T2``
    path (``gemm_cuda.cu:1206-1232``), never the M <= 32 split-K path.
    ``c0``: BASELINE config 0 (X [1374, 1024] ~ N(0,1), W 1024 -> 4096, g128, seed 0).
    """
    from oracle import awq
    c = {}
    N, K, G = 512, 1024, 128
    rng = np.random.default_rng(12)
    q = rng.integers(0, 16, size=(N, K), dtype=np.int32)
    zeros = rng.integers(0, 16, size=(N, K // G)).astype(np.float32)
    mult = 2.0 ** rng.integers(-6, 7, size=(N, K // G))
    scales = np.maximum(np.abs(rng.standard_normal((N, K // G))) * 0.02 * mult, 1e-4).astype(np.float16)
    gpad = awq.calculate_zeros_width(K, G) * 8
    st = np.zeros((gpad, N), np.float16)
    st[: K // G] = scales.T
    szt = np.zeros((gpad, N), np.float16)
    szt[: K // G] = (-(scales.astype(np.float32) * zeros)).astype(np.float16).T
    c["eye"] = dict(x=np.eye(K, dtype=np.float16), qweight=awq.pack_intweight(q), scales=st, scaled_zeros=szt)
    lin = awq.make_quantized_linear(4096, 1024, 128, seed=0, bias=False)
    x = np.random.default_rng(0).standard_normal((1374, 1024)).astype(np.float16)
    c["c0"] = dict(x=x, qweight=lin["qweight"], scales=lin["scales"], scaled_zeros=lin["scaled_zeros"])
    return c


def bf16_pin_cases():
    """Inputs of the bf16 pins: the reference's bf16 instantiation of
    gemm_forward_cuda_new / gemv_forward_cuda_new (``dispatch_utils.cuh:7-17``).
    bf16 tensors are held as float32 arrays of bf16 values (numpy has no bf16).

    ``eye``: as :func:`gemm_pin_cases`' eye case in bf16 (A = I, M = K = 1024,
    N = 512, scales over 2^-6 .. 2^6 times the config-0 distribution, all 16
    nibble values and zero points): C = deq_bf16(W)^T bit for bit (one exact
    product per output, fp32 accumulation, an exact bf16 store).
    ``lin``: N = 512, K = 1024, g128 bf16 weights; X [300, 1024] ~ N(0, 1) in
    bf16 for the GEMM (``gemm_w4a16_T2``), its first 1 and 5 rows for the GEMV.
    """
    from oracle import awq
    c = {}
    N, K, G = 512, 1024, 128
    rng = np.random.default_rng(13)
    q = rng.integers(0, 16, size=(N, K), dtype=np.int32)
    zeros = rng.integers(0, 16, size=(N, K // G)).astype(np.float64)
    mult = 2.0 ** rng.integers(-6, 7, size=(N, K // G))
    scales = awq.bf16_round(np.maximum(np.abs(rng.standard_normal((N, K // G))) * 0.02 * mult, 1e-4))
    gpad = awq.calculate_zeros_width(K, G) * 8
    st = np.zeros((gpad, N), np.float32)
    st[: K // G] = scales.T
    szt = np.zeros((gpad, N), np.float32)
    szt[: K // G] = awq.bf16_round(-(scales.astype(np.float64) * zeros)).T
    c["eye"] = dict(x=np.eye(K, dtype=np.float32), qweight=awq.pack_intweight(q), scales=st, scaled_zeros=szt)
    lin = awq.make_quantized_linear_bf16(N, K, G, seed=14, bias=False)
    x = awq.bf16_round(np.random.default_rng(15).standard_normal((300, K)))
    c["lin"] = dict(x=x, qweight=lin["qweight"], scales=lin["scales"], scaled_zeros=lin["scaled_zeros"])
    return c


def generate_bf16_pins(ref, dev="cuda"):
    """Outputs (uint16 bf16 bit patterns) of the reference kernels on
    :func:`bf16_pin_cases`."""
    from oracle import awq
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).to(dev)
    qw = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    bits = lambda y: awq.bf16_bits(y.float().cpu().numpy())
    c = bf16_pin_cases()
    out = {}
    d = c["eye"]
    out["eye_y"] = bits(ref.gemm_forward_cuda_new(bf(d["x"]), qw(d["qweight"]), bf(d["scales"]),
                                                  bf(d["scaled_zeros"])))
    d = c["lin"]
    out["gemm_y"] = bits(ref.gemm_forward_cuda_new(bf(d["x"]), qw(d["qweight"]), bf(d["scales"]),
                                                   bf(d["scaled_zeros"])))
    K, N = d["x"].shape[1], d["qweight"].shape[0] * 4
    for m in (1, 5):
        y = ref.gemv_forward_cuda_new(bf(d["x"][:m]), qw(d["qweight"]), bf(d["scales"]), bf(d["scaled_zeros"]), m, N,
                                      K, 128)
        out[f"gemv_m{m}_y"] = bits(y)
    torch.cuda.synchronize()
    return out


def generate_gemm_pins(ref, dev="cuda"):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    c = gemm_pin_cases()
    out = {}
    d = c["eye"]
    out["eye_y"] = ref.gemm_forward_cuda_new(t(d["x"]), t(d["qweight"]), t(d["scales"]),
                                             t(d["scaled_zeros"])).cpu().numpy()
    d = c["c0"]
    y = ref.gemm_forward_cuda_new(t(d["x"]), t(d["qweight"]), t(d["scales"]), t(d["scaled_zeros"]))
    out["c0_rows_y"] = y[torch.tensor(C0_ROWS, device=dev)].cpu().numpy()
    torch.cuda.synchronize()
    return out


def generate(ref, dev="cuda"):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    out = {}
    c = cases()
    for name in ("gemm_a", "gemm_b"):
        d = c[name]
        y = ref.gemm_forward_cuda_new(t(d["x"]), t(d["qweight"]), t(d["scales"]), t(d["scaled_zeros"]))
        out[f"{name}_y"] = y.cpu().numpy()
    d = c["gemm_a"]
    for m in (1, 7):
        K, N = d["x"].shape[1], d["qweight"].shape[0] * 4
        y = ref.gemv_forward_cuda_new(t(d["x"][:m]), t(d["qweight"]), t(d["scales"]), t(d["scaled_zeros"]), m, N, K,
                                      128)
        out[f"gemv_m{m}_y"] = y.cpu().numpy()
    d = c["w8a8"]
    o = torch.empty(200, 256, dtype=torch.float16, device=dev)
    ref.w8a8_gemm_forward_cuda(t(d["a"]), t(d["w"]), t(d["ws"]), t(d["as_"]), o)
    out["w8a8_y"] = o.cpu().numpy()
    o2 = torch.empty(200, 256, dtype=torch.float16, device=dev)
    ref.w8a8_gemm_fuse_bias_forward_cuda(t(d["a"]), t(d["w"]), t(d["ws"]), t(d["as_"]), o2, t(d["bias"]))
    out["w8a8_bias_y"] = o2.cpu().numpy()
    x = t(c["quant"]["x"])
    q = torch.empty(x.shape, dtype=torch.int8, device=dev)
    s = torch.empty(x.shape[0], dtype=torch.float16, device=dev)
    ref.invoke_quant(q, x, s)
    out["quant_q"], out["quant_s"] = q.cpu().numpy(), s.cpu().numpy()
    d = c["ln"]
    x = t(d["x"])
    q = torch.empty(x.shape, dtype=torch.int8, device=dev)
    s = torch.empty(x.shape[0], dtype=torch.float16, device=dev)
    ref.rms_norm_general(q, x, t(d["w"]), t(d["b"]), s, 1e-6, True)
    out["ln_q"], out["ln_s"] = q.cpu().numpy(), s.cpu().numpy()
    q2 = torch.empty(x.shape, dtype=torch.int8, device=dev)
    s2 = torch.tensor([20.0], dtype=torch.float16, device=dev)
    ref.rms_norm_general(q2, x, t(d["w"]), t(d["b"]), s2, 1e-6, False)
    out["ln_tensor_q"] = q2.cpu().numpy()
    x = t(c["gelu"]["x"])
    q = torch.empty(x.shape, dtype=torch.int8, device=dev)
    s = torch.empty(x.shape[0], dtype=torch.float16, device=dev)
    tmp = torch.empty(x.shape, dtype=torch.float16, device=dev)
    ref.gelu_and_quant(q, x, s, tmp)
    out["gelu_q"], out["gelu_s"], out["gelu_tmp"] = q.cpu().numpy(), s.cpu().numpy(), tmp.cpu().numpy()
    d = c["rope"]
    for tr in (False, True):
        y = ref.fused_rope_with_pos_forward_func(t(d["x"]), t(d["freqs"]), tr)
        out[f"rope_y_{int(tr)}"] = y.contiguous().cpu().numpy()
    torch.cuda.synchronize()
    return out


def time_reference(ref, dev="cuda"):
    """CUDA-event timings of the reference kernels at the benchmark shapes."""
    from oracle import awq

    def timeit(fn, iters=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / iters / 1e3

    res = {}
    for (M, N, K) in [(1374, 4096, 1024), (43968, 3072, 1024), (43968, 1024, 1024), (43968, 4096, 1024),
                      (43968, 1024, 4096)]:
        lin = awq.make_quantized_linear(N, K, 128, seed=1, bias=False)
        qw, s, z = (torch.from_numpy(lin[k]).to(dev) for k in ("qweight", "scales", "scaled_zeros"))
        x = torch.randn(M, K, dtype=torch.float16, device=dev)
        sec = timeit(lambda: ref.gemm_forward_cuda_new(x, qw, s, z))
        res[f"gemm_w4a16 M={M} N={N} K={K}"] = (sec * 1e6, 2 * M * N * K / sec / 1e12)
    lin = awq.make_quantized_linear(4096, 1024, 128, seed=1, bias=False)
    qw, s, z = (torch.from_numpy(lin[k]).to(dev) for k in ("qweight", "scales", "scaled_zeros"))
    x1 = torch.randn(1, 1024, dtype=torch.float16, device=dev)
    sec = timeit(lambda: ref.gemv_forward_cuda_new(x1, qw, s, z, 1, 4096, 1024, 128), iters=200)
    res["gemv_w4a16 m=1 N=4096 K=1024"] = (sec * 1e6, 2 * 4096 * 1024 / sec / 1e12)
    M, N, K = 87936, 4096, 1024
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev)
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
    ws = torch.rand(N, device=dev).half()
    as_ = torch.rand(M, device=dev).half()
    o = torch.empty(M, N, dtype=torch.float16, device=dev)
    sec = timeit(lambda: ref.w8a8_gemm_forward_cuda(a, w, ws, as_, o))
    res[f"w8a8_gemm M={M} N={N} K={K}"] = (sec * 1e6, 2 * M * N * K / sec / 1e12)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "ref_cuda_golden.npz"))
    ap.add_argument("--time", action="store_true")
    ap.add_argument("--gemm-pins", default=None, help="write only the GEMM pin fixture to this path")
    ap.add_argument("--bf16-pins", default=None, help="write only the bf16 GEMM / GEMV pin fixture to this path")
    a = ap.parse_args()
    from oracle import build_ref
    ref = build_ref.load()
    if a.bf16_pins:
        out = generate_bf16_pins(ref)
        np.savez_compressed(a.bf16_pins, **out)
        print("wrote", a.bf16_pins, {k: v.shape for k, v in out.items()})
        return
    if a.gemm_pins:
        out = generate_gemm_pins(ref)
        np.savez_compressed(a.gemm_pins, **out)
        print("wrote", a.gemm_pins, {k: v.shape for k, v in out.items()})
        return
    out = generate(ref)
    np.savez_compressed(a.out, **out)
    print("wrote", a.out, {k: v.shape for k, v in out.items()})
    if a.time:
        for k, (us, tf) in time_reference(ref).items():
            print(f"REF {k}: {us:.1f} us  {tf:.1f} TFLOP/s")


if __name__ == "__main__":
    main()
