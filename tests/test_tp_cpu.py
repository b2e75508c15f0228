"""Tensor-parallel partition on CPU with two `gloo` ranks: each rank computes
its rows of layer 0's linear layers and of the classifier with the scalar
oracle (full K, the reference's kernels), the ranks all-gather the parts,
and the gathered vectors must equal the single-rank matvecs bit for bit —
the property that makes nrc_tp_ctx_new bit-identical to one GPU. Also the
shards tile the model exactly."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MODELS = ["tiny_llama_q8", "tiny_qwen3"]  # two KV heads: a whole KV group per rank


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tensors(orc, blob):
    m = orc.model(blob)
    data_off = int.from_bytes(blob[168:176].tobytes(), "little")
    out = {}
    for kind, layer, dtype, off, size, rows, cols in m.tensors():
        out[(kind, layer)] = (dtype, blob[data_off + off:data_off + off + size], rows, cols)
    return out


FMT = {1: ("q8_0", 34, 32), 2: ("q4k", 144, 256), 3: ("q6k", 210, 256)}


def _matvec_rows(orc, t, r0, n, x):
    dtype, data, rows, cols = t
    fmt, bb, blk = FMT[dtype]
    rb = cols // blk * bb
    part = np.ascontiguousarray(data[r0 * rb:(r0 + n) * rb])
    xq = orc.q8_quantize(x) if fmt == "q8_0" else orc.quantize_q8k(x)
    return orc.matvec(fmt, part, xq, n, cols)


def _rank(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    from nightrun_b200 import tp
    from nightrun_b200.configs import CONFIGS, MODEL_SEED
    from oracle import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        orc = O.get()
        orc.set_mode(False)
        ok = []
        for name in MODELS:
            cfg = CONFIGS[name]
            blob = orc.synth_nrm(cfg, MODEL_SEED)
            T = _tensors(orc, blob)
            sh = tp.shard(cfg, world, rank)
            _, _, h0, nh, kv0, nkv, d0, dn, f0, fn, v0, vn = sh
            hd = cfg["head_dim"]
            x = np.random.default_rng(7).standard_normal(cfg["dim"]).astype(np.float32)
            xa = np.random.default_rng(8).standard_normal(cfg["n_heads"] * hd).astype(np.float32)
            xf = np.random.default_rng(9).standard_normal(cfg["ffn_dim"]).astype(np.float32)
            jobs = [((11, 0), h0 * hd, nh * hd, x), ((12, 0), kv0 * hd, nkv * hd, x), ((13, 0), kv0 * hd, nkv * hd, x),
                    ((14, 0), d0, dn, xa), ((16, 0), f0, fn, x), ((17, 0), f0, fn, x), ((18, 0), d0, dn, xf),
                    ((3, 0) if (3, 0) in T else (1, 0), v0, vn, x)]
            for key, r0, n, xin in jobs:
                mine = torch.from_numpy(_matvec_rows(orc, T[key], r0, n, xin))
                parts = [torch.empty_like(mine) for _ in range(world)]
                dist.all_gather(parts, mine)
                got = torch.cat(parts).numpy()
                full = _matvec_rows(orc, T[key], 0, T[key][2], xin)
                ok.append((name, key, got.tobytes() == full.tobytes()))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_two_rank_partition_bit_identical():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for _ in range(world):
        rank, ok = q.get(timeout=5)
        bad = [o for o in ok if not o[2]]
        assert not bad, f"rank {rank}: {bad}"


@pytest.mark.parametrize("name", ["llama1b_q8", "llama3b_q4km", "qwen3_4b_q4km", "granite3b_q4km"])
@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_shards_tile_the_model(name, n):
    sys.path.insert(0, ROOT)
    from nightrun_b200 import tp
    from nightrun_b200.configs import CONFIGS
    cfg = CONFIGS[name]
    shards = [tp.shard(cfg, n, r) for r in range(n)]
    for idx, total in ((2, cfg["n_heads"]), (4, cfg["n_kv_heads"]), (6, cfg["dim"]), (8, cfg["ffn_dim"]),
                       (10, cfg["vocab"])):
        covered = []
        for s in shards:
            covered += list(range(s[idx], s[idx] + s[idx + 1]))
        assert covered == list(range(total)), (name, n, idx)
    gqa = cfg["n_heads"] // cfg["n_kv_heads"]
    for s in shards:  # query heads of a rank are exactly those of its KV groups
        assert s[2] == s[4] * gqa and s[3] == s[5] * gqa
