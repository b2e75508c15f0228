"""Tensor parallelism over NCCL (nrc_tp_ctx_new) on 2 or more GPUs of one box:
prefill, host-driven decode and device-side generation bit-identical to a
single-GPU context (every output row is computed whole by one rank; ranks
exchange activations, never partial sums). Skipped with fewer GPUs."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("name", ["tiny_llama_q8", "tiny_qwen3", "llama1b_q8", "llama3b_q4km"])
def test_tensor_parallel_bit_identical(tmp_path, name):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    out = str(tmp_path / "tp")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(29500 + os.getpid() % 1000),
           os.path.join(ROOT, "tests", "tp_worker.py"), name, "12", out]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = [json.load(open(f"{out}.{k}.json")) for k in range(world)]
    assert res[0]["tokens_equal"], res[0]
    assert res[0]["logits_equal"], res[0]
    # The shards tile the model: heads, rows and vocabulary each split evenly.
    assert [r_["shard"][1] for r_ in res] == list(range(world))
