#!/usr/bin/env python
"""Benchmark of the quantized forward path on B200 (config 0 decode, b = 1).

A step is one greedy decode token of config 0 (Llama-3.2-1B architecture,
all linear weights Q8_0, seeded synthetic weights) after a 64-token prompt;
the timed steps sit at positions 64+W .. 64+W+K-1.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line (rank 0). `value` is device-resident throughput (graph
replays, CUDA events on the library's stream, max over ranks); `e2e` goes
through the public API with host buffers every step (token H2D, logits D2H).
N > 1 runs independent sequences per GPU (data parallel, weak scaling).
`--impl reference` times the CPU restatement of the reference's AVX2 path.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from nightrun_b200.configs import CONFIGS, MODEL_SEED, prompt_ids  # noqa: E402

METRIC = "decode tokens/s (b=1 and batched); quant-GEMV HBM GB/s vs ~8 TB/s peak"
CFG_NAME = "llama1b_q8"
PROMPT = 64
# Published CPU number of the reference for this metric and model (docs/baseline-x86.md:23).
PUBLISHED_TOKS = 21.7
WORKLOAD = ("config0: Llama-3.2-1B architecture, all linear weights Q8_0, random-init synthetic weights; "
            "64-token seed-uniform prompt, then greedy decode at b=1")


def model_bytes(cfg):
    """Algorithmic bytes per decode token: packed weights read once + KV read at mean position."""
    dim, L, ffn, vocab = cfg["dim"], cfg["n_layers"], cfg["ffn_dim"], cfg["vocab"]
    att, kv = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    per_layer = dim * att + 2 * dim * kv + att * dim + 3 * dim * ffn
    w = (per_layer * L + vocab * dim) * 34 // 32
    norms = (2 * L + 1) * dim * 4
    return w + norms, L * 2 * kv * 2  # weight bytes, KV bytes per position


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.path = os.path.join("/tmp", f"nrc_clocks_{os.getpid()}_{gpu}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.12)
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                    pw.append(float(parts[3]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.remove(self.path)
        loaded = [s for s, p in zip(sm, pw) if p > 250.0] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm), "samples_under_load": len(loaded)}


def launches_per_step(cfg):
    # embed + per layer (QKV, attention with RoPE/KV append fused, wo, gate/up, down) + classifier + finish
    return 1 + cfg["n_layers"] * 5 + 2


def cpu_decode(blob, cfg, steps, warmup, threads):
    """The reference's AVX2 path (CPU restatement) on this host: tokens/s of greedy decode."""
    from oracle import oracle as O
    orc = O.get()
    orc.set_mode(True)  # AVX2 + F16C kernels, as the reference runs on x86
    orc.pool_start(threads)
    m = orc.model(blob)
    c = m.ctx(PROMPT + warmup + steps + 8)
    logits = c.prefill(np.array(prompt_ids(PROMPT, cfg["vocab"]), np.uint32))
    nxt = int(np.argmax(logits))
    for _ in range(warmup):
        nxt = int(np.argmax(c.forward(nxt)))
    t0 = time.perf_counter()
    for _ in range(steps):
        nxt = int(np.argmax(c.forward(nxt)))
    dt = time.perf_counter() - t0
    return steps / dt, dt


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle as O
    cfg = CONFIGS[CFG_NAME]
    threads = os.cpu_count()
    blob = O.get().synth_nrm(cfg, MODEL_SEED, threads=threads)
    tps, dt = cpu_decode(blob, cfg, args.steps, args.warmup, threads)
    sample = (f"config0 greedy decode: {PROMPT}-token prompt prefilled, {args.warmup} warm-up + {args.steps} "
              f"timed decode tokens on {threads} host threads (C++ restatement of the reference AVX2 path)")
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": tps / PUBLISHED_TOKS,
            "dtype": "q8_0 (i8 dot, f32)", "data": "synthetic (seeded random-init weights, seed-uniform prompt)",
            "config": {"workload": WORKLOAD, "prompt": PROMPT, "batch": 1},
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) of one classifier-shape launch, from the ncu capture
# in profiles/gemv_lr_q8_0_classifier_128256x2048_n1.md (same command shape).
CLASSIFIER_TRAFFIC = 282_699_520


def gemv_roofline(torch, K, rows, cols, reps, stream):
    """Standalone Q8_0 GEMV on the classifier shape (the largest decode launch)."""
    from nightrun_b200 import kernels
    nb = rows * cols // 32
    g = torch.Generator(device="cuda").manual_seed(1)
    w = torch.randint(-127, 128, (nb, 34), dtype=torch.int16, device="cuda", generator=g).to(torch.int8)
    w = w.view(torch.uint8)
    w[:, 0] = 0x00
    w[:, 1] = 0x20  # f16 scale 2^-7
    w = w.contiguous().view(-1)
    x = torch.randn(cols, device="cuda")
    xq = torch.empty(cols // 32 * 34, dtype=torch.uint8, device="cuda")
    y = torch.empty(rows, device="cuda")
    kernels.quantize(x, xq, stream=stream)
    for _ in range(3):
        kernels.matvec_q8(y, w, xq, rows, cols, stream=stream)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(reps):
        kernels.matvec_q8(y, w, xq, rows, cols, stream=stream)
    ev1.record(stream)
    ev1.synchronize()
    kernels.sync_check(stream)
    ms = ev0.elapsed_time(ev1) / reps
    nbytes = nb * 34 + cols // 32 * 34 + rows * 4
    del w
    return nbytes, ms


def max_over_ranks_of(v, world, device):
    """The slowest rank's time: every timed region is reported as the max over
    ranks (an all-reduce MAX on `device`; the process group must be up)."""
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_tokens_per_s(ms_max, steps, world):
    """Whole-job throughput of `world` independent replicas that each decoded
    `steps` tokens, timed by the slowest rank."""
    return world * steps / (ms_max / 1000.0)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    from nightrun_b200 import Model
    cfg = CONFIGS[CFG_NAME]
    W, Kst = args.warmup, args.steps
    sampler = ClockSampler(local_rank)
    model = Model.synth(cfg, MODEL_SEED, device=local_rank)
    ctx = model.ctx(PROMPT + W + Kst + 8)
    stream = torch.cuda.ExternalStream(ctx.stream_handle())
    prompt = np.array(prompt_ids(PROMPT, cfg["vocab"]), np.uint32)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        return max_over_ranks_of(v, world, "cuda")

    sampler.start()
    # ---- device-resident decode (graph replay per token)
    ctx.prefill(prompt)
    ctx.decode_async(W)
    ctx.sync()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    ctx.decode_async(Kst)
    ev1.record(stream)
    ctx.sync()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    value = job_tokens_per_s(ms, Kst, world)

    # ---- end to end through the public API: host token in, host logits out, every step
    ctx.reset()
    vocab = cfg["vocab"]
    logits_host = torch.empty(vocab, dtype=torch.float32, pin_memory=True)
    next_host = torch.empty(1, dtype=torch.int32, pin_memory=True)
    import ctypes as C
    lp, npt = C.c_void_p(logits_host.data_ptr()), C.c_void_p(next_host.data_ptr())
    ctx.prefill(prompt)
    tok = ctx.next_token
    for _ in range(W):
        ctx.forward_into(tok, lp, npt)
        tok = int(next_host.item())
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(Kst):
        ctx.forward_into(tok, lp, npt)
        tok = int(next_host.item())
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = job_tokens_per_s(e2e_ms, Kst, world)

    # ---- dominant kernel: Q8_0 GEMV on the classifier shape (vocab x dim)
    gstream = torch.cuda.Stream()
    gbytes, gms = gemv_roofline(torch, None, vocab, cfg["dim"], 20, gstream)
    clocks = sampler.stop()
    hbm, hbm_kind = peaks()
    achieved = gbytes / (gms / 1000.0) / 1e9
    wbytes, kv_per_pos = model_bytes(cfg)
    mean_pos = PROMPT + W + Kst / 2.0
    step_bytes = wbytes + kv_per_pos * mean_pos
    step_gbs = step_bytes * (value / world) / 1e9

    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": Kst, "warmup": W,
            "ms_per_step": ms / Kst, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / PUBLISHED_TOKS, "dtype": "q8_0 (i8 dot, f32)",
            "data": "synthetic (seeded random-init weights, seed-uniform prompt)",
            "config": {"workload": WORKLOAD, "prompt": PROMPT, "batch": 1,
                       "parallelism": f"dp{world} (independent sequences)" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (1.31 GB of weights streamed per step)"},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": vocab * 4 + 8},
            "gpu_launches": launches_per_step(cfg) * Kst,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": CLASSIFIER_TRAFFIC,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch of the same "
                                           "shape (profiles/gemv_lr_q8_0_classifier_128256x2048_n1.md)",
                         "kernel": f"gemv_lr_kernel<1> Q8_0 {vocab}x{cfg['dim']} (classifier), {gms * 1000:.1f} us/launch",
                         "peak_kind": hbm_kind,
                         "algorithmic_bytes_per_launch": gbytes},
            "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_gbs, "frac": step_gbs / hbm},
            "clocks": clocks}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        blob = model.export()
        threads = os.cpu_count()
        steps = args.cpu_steps
        tps, dt = cpu_decode(blob, cfg, steps, 2, threads)
        line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": f"config0 greedy decode, {PROMPT}-token prompt then {steps} tokens "
                                          f"({dt:.1f} s) with the C++ restatement of the reference AVX2 path"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    model.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=96)
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
