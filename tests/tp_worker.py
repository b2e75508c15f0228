"""One rank of a tensor-parallel run (launched by tests/test_gpu_tp.py through
torch.distributed.run): every rank builds the same seeded model on its GPU,
joins an NCCL group through nrc_tp_ctx_new, prefills and decodes; rank 0
also runs the same steps on a single-GPU context and records whether every
logit and token matched bit for bit."""
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import nightrun_b200 as NB  # noqa: E402
from nightrun_b200.configs import CONFIGS, MODEL_SEED, prompt_ids  # noqa: E402


def main():
    name, steps, out = sys.argv[1], int(sys.argv[2]), sys.argv[3]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo")
    cfg = CONFIGS[name]
    uid = [NB.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    m = NB.Model.synth(cfg, MODEL_SEED, device=rank)
    c = m.ctx(160, tp=(world, rank, uid[0]))
    ids = prompt_ids(40, cfg["vocab"])
    got = [c.prefill(ids)]
    toks = [c.next_token]
    for _ in range(steps):
        got.append(c.forward(toks[-1]))
        toks.append(c.next_token)
    gen = [int(t) for t in c.generate(toks[-1], 8)]
    shard = c.shard()
    res = {"rank": rank, "shard": shard}
    if rank == 0:
        r = m.ctx(160)
        ref = [r.prefill(ids)]
        rt = [r.next_token]
        for _ in range(steps):
            ref.append(r.forward(rt[-1]))
            rt.append(r.next_token)
        rgen = [int(t) for t in r.generate(rt[-1], 8)]
        res["logits_equal"] = all(a.tobytes() == b.tobytes() for a, b in zip(got, ref))
        res["max_abs"] = max(float(np.max(np.abs(a - b))) for a, b in zip(got, ref))
        res["tokens_equal"] = toks == rt and gen == rgen
        r.close()
    c.close()
    m.close()
    with open(f"{out}.{rank}.json", "w") as f:
        json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
