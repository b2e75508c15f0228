"""Quantized GEMV/GEMM sweep (config 1): achieved HBM GB/s of the kernel-level
matvec/matmul entry points on device-resident random weights.

    python -m nightrun_b200.bench_gemv                       # full config-1 sweep, JSON lines
    python -m nightrun_b200.bench_gemv --fmt q8_0 --rows 128256 --cols 2048 --n 1 --reps 3

Algorithmic bytes per launch = packed weight bytes + activation blocks + f32 outputs.
Consecutive launches use different weight copies (more than L2 together); the
timed launches are replayed as one CUDA graph, so CUDA events measure the GPU
rather than the host's per-call work.
"""
import argparse
import json

import torch

from . import kernels

SHAPES = [(2048, 2048), (8192, 2048), (2048, 8192), (128256, 2048), (9728, 2560)]
BLOCK = {"q8_0": (32, 34), "q4k": (256, 144), "q6k": (256, 210)}


def random_weights(fmt, rows, cols, gen):
    """Valid random blocks: random quants, finite f16 scales."""
    per, nbytes = BLOCK[fmt]
    nb = rows * cols // per
    w = torch.randint(0, 256, (nb, nbytes), dtype=torch.int16, device="cuda", generator=gen).to(torch.uint8)
    if fmt == "q8_0":
        w[:, 0], w[:, 1] = 0x00, 0x20            # d = 2^-7
    elif fmt == "q4k":
        w[:, 0], w[:, 1], w[:, 2], w[:, 3] = 0x00, 0x20, 0x00, 0x1C   # d, dmin
    else:
        w[:, 208], w[:, 209] = 0x00, 0x20
    return w.contiguous().view(-1)


def run(fmt, rows, cols, n, reps, stream):
    gen = torch.Generator(device="cuda").manual_seed(rows * 31 + cols)
    w = random_weights(fmt, rows, cols, gen)
    x = torch.randn(n * cols, device="cuda", generator=gen)
    per = BLOCK[fmt][0]
    xb = 34 if fmt == "q8_0" else 292
    xq = torch.empty(n * cols // per * xb, dtype=torch.uint8, device="cuda")
    (kernels.quantize if fmt == "q8_0" else kernels.quantize_q8k)(x, xq, stream=stream)
    y = torch.empty(n * rows, device="cuda")
    fn = {"q8_0": kernels.matmul_q8, "q4k": kernels.matmul_q4k, "q6k": kernels.matmul_q6k}[fmt]
    # Rotate over weight copies larger than L2 (126 MB) together, so every
    # launch streams its weights from HBM.
    copies = [w] + [w.clone() for _ in range(max(0, (160 << 20) // w.numel()))]
    def launches():
        for i in range(reps):
            fn(y, copies[i % len(copies)], xq, rows, cols, n, stream=stream)

    for i in range(3):
        fn(y, copies[i % len(copies)], xq, rows, cols, n, stream=stream)
    torch.cuda.synchronize()
    # The timed launches as one CUDA graph: the events then measure the GPU,
    # not the host's per-call work (scratch allocation, tensor-map encoding,
    # two launches), which for the small shapes takes longer than the kernels.
    timing = "graph"
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="relaxed"):
            launches()

        def replay():
            with torch.cuda.stream(stream):
                g.replay()
    except Exception:  # capture unavailable: time the eager launches
        timing = "eager"
        replay = launches
    replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    replay()
    e1.record(stream)
    e1.synchronize()
    kernels.sync_check(stream)
    us = e0.elapsed_time(e1) * 1000.0 / reps
    nbytes = w.numel() + xq.numel() + y.numel() * 4
    return {"fmt": fmt, "rows": rows, "cols": cols, "n": n, "us": us, "bytes": nbytes,
            "gbs": nbytes / us / 1e3, "int8_tops": 2.0 * rows * cols * n / us / 1e6, "timing": timing}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--fmt", default=None)
    ap.add_argument("--rows", type=int, default=None)
    ap.add_argument("--cols", type=int, default=None)
    ap.add_argument("--n", type=int, default=None)
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args()
    stream = torch.cuda.Stream()
    if args.fmt:
        print(json.dumps(run(args.fmt, args.rows, args.cols, args.n or 1, args.reps, stream)))
        return
    for fmt in ("q8_0", "q4k", "q6k"):
        for rows, cols in SHAPES:
            for n in (1, 8, 64):
                print(json.dumps(run(fmt, rows, cols, n, args.reps, stream)), flush=True)


if __name__ == "__main__":
    main()
