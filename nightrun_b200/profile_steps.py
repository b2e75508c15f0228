"""Decode steps bracketed by cudaProfilerStart/Stop, for ncu launch lists
(`ncu --profile-from-start off ...`):

    python -m nightrun_b200.profile_steps c0    # config 0, exact mode: 2 decode steps at positions 68-69
    python -m nightrun_b200.profile_steps c0f   # the same in the tolerance mode
    python -m nightrun_b200.profile_steps c4    # config 4: one decode step of 256 sequences (128-token prompts)
"""
import sys

import numpy as np
import torch

from . import Model
from .configs import CONFIGS, MODEL_SEED, prompt_ids


def main(which):
    if which in ("c0", "c0f"):
        cfg = CONFIGS["llama1b_q8"]
        m = Model.synth(cfg, MODEL_SEED)
        c = m.ctx(256)
        c.set_mode(1 if which == "c0f" else 0)
        c.prefill(np.array(prompt_ids(64, cfg["vocab"]), np.uint32))
        c.decode_async(4)
        c.sync()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        c.decode_async(2)
        c.sync()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    elif which == "c4":
        cfg = CONFIGS["granite3b_q4km"]
        m = Model.synth(cfg, MODEL_SEED)
        b = m.batch(160, 256)
        b.prefill([prompt_ids(128, cfg["vocab"], seed=MODEL_SEED + 11 + i) for i in range(256)])
        b.decode_async(2)
        b.sync()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        b.decode_async(1)
        b.sync()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    else:
        raise SystemExit(f"unknown workload {which!r}: c0, c0f or c4")
    print("ok", which)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "c0")
