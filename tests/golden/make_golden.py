"""Generate tests/golden/config0_greedy.npz with the CPU oracle (scalar path).

Config 0 (Llama-3.2-1B architecture, all Q8_0, seeded synthetic weights):
prefill a 64-token seed-uniform prompt, then greedy-decode 128 tokens. The
fixture holds the prompt, the scalar reference's greedy tokens, the logits
after the prefill, the data CRC of the synthetic weights and the top-2 logit
gap of every step (near-ties explain any divergence). It is checked on the
GPU by tests/test_gpu_model.py::test_config0_greedy_matches_golden.

    python tests/golden/make_golden.py [--threads N]
"""
import argparse
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from nightrun_b200.configs import CONFIGS, MODEL_SEED, prompt_ids  # noqa: E402
from oracle import oracle as O  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    ap.add_argument("--steps", type=int, default=128)
    args = ap.parse_args()
    orc = O.get()
    orc.set_mode(False)  # scalar kernels: the bit-exact reference
    orc.pool_start(args.threads)
    cfg = CONFIGS["llama1b_q8"]
    t0 = time.time()
    blob = orc.synth_nrm(cfg, MODEL_SEED, threads=args.threads)
    data_off = int.from_bytes(blob[168:176].tobytes(), "little")
    data_crc = orc.crc32(blob[data_off:])
    print(f"synth {blob.size / 1e9:.2f} GB in {time.time() - t0:.1f}s, crc {data_crc:#x}", flush=True)
    m = orc.model(blob)
    c = m.ctx(256)
    prompt = np.array(prompt_ids(64, cfg["vocab"]), np.uint32)
    t0 = time.time()
    logits = c.prefill(prompt)
    print(f"prefill {time.time() - t0:.1f}s", flush=True)
    logits_prefill = logits.copy()
    toks, gaps = [], []
    t0 = time.time()
    for i in range(args.steps):
        top = np.partition(logits, -2)[-2:]
        gaps.append(float(top.max() - top.min()))
        nxt = int(np.argmax(logits))
        toks.append(nxt)
        if i + 1 < args.steps:
            logits = c.forward(nxt)
    print(f"decode {args.steps} in {time.time() - t0:.1f}s; min top-2 gap {min(gaps):.3e}", flush=True)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "config0_greedy.npz")
    np.savez_compressed(out, seed=np.uint64(MODEL_SEED), data_crc=np.uint32(data_crc), prompt=prompt,
                        tokens=np.array(toks, np.uint32), logits_prefill=logits_prefill.astype(np.float32),
                        gaps=np.array(gaps, np.float32))
    print("wrote", out)


if __name__ == "__main__":
    main()
