"""GPU parity at the full sizes of the benchmark configurations.

* Config 1: every matvec / matmul shape of the standalone sweep
  ([2048x2048, 8192x2048, 2048x8192, 128256x2048, 9728x2560] x
  {Q8_0, Q4_K, Q6_K} x N in {1, 8, 64}) bit-identical to the reference's
  scalar kernels (crates/nr-tensor/src/kernels.rs:36-143,
  crates/nr-tensor/src/kquant.rs:536-639). The weight blocks are seeded random
  bytes with finite f16 scales: every quant pattern, not only the ones a
  rounding quantizer produces.
* Configs 2, 3 and 4 at full size (Llama-3.2-3B, Qwen3-4B and Granite-4.1-3B
  architectures, Q4_K/Q6_K mix): one 64-token prefill chunk plus 8 decode
  steps, logits and KV rows bit-identical to the scalar oracle
  (crates/nr-model/src/infer.rs:510-750).
* Attention past the config-3 context length (2,304 positions) on a small
  Qwen3 model with head_dim 128 (infer.rs:553-572).
"""
import os

import numpy as np
import pytest
import torch

from nightrun_b200.configs import CONFIGS, MODEL_SEED, prompt_ids

pytestmark = pytest.mark.gpu

CONFIG1_SHAPES = [(2048, 2048), (8192, 2048), (2048, 8192), (128256, 2048), (9728, 2560)]
BLOCK = {"q8_0": (32, 34), "q4k": (256, 144), "q6k": (256, 210)}


def random_blocks(fmt, nblocks, seed):
    """Seeded random weight blocks of `fmt` with finite, positive f16 scales."""
    r = np.random.default_rng(seed)
    _, nbytes = BLOCK[fmt]
    b = r.integers(0, 256, (nblocks, nbytes), dtype=np.uint8)

    def f16(lo, hi):
        return r.uniform(lo, hi, nblocks).astype(np.float16).view(np.uint8).reshape(nblocks, 2)

    if fmt == "q8_0":
        b[:, 0:2] = f16(1e-4, 2e-3)
        q = b[:, 2:].view(np.int8)
        q[q == -128] = -127  # q8::quantize never writes -128
    elif fmt == "q4k":
        b[:, 0:2] = f16(1e-4, 2e-3)
        b[:, 2:4] = f16(1e-5, 1e-3)
    else:
        b[:, 208:210] = f16(1e-4, 2e-3)
    return np.ascontiguousarray(b)


def acts(orc, fmt, cols, batch, seed):
    x = np.random.default_rng(seed).standard_normal(cols * batch).astype(np.float32)
    return orc.q8_quantize(x) if fmt == "q8_0" else orc.quantize_q8k(x)


@pytest.fixture(scope="module")
def K():
    from nightrun_b200 import kernels
    return kernels


@pytest.fixture(scope="module")
def pool(orc):
    orc.pool_start(os.cpu_count() or 8)
    return orc


def to_dev(a):
    return torch.from_numpy(np.frombuffer(np.ascontiguousarray(a).tobytes(), np.uint8).copy()).cuda()


@pytest.mark.parametrize("fmt", ["q8_0", "q4k", "q6k"])
@pytest.mark.parametrize("shape", CONFIG1_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_config1_full_shapes_bit_exact(K, pool, fmt, shape):
    orc = pool
    orc.set_mode(False)
    rows, cols = shape
    blk, _ = BLOCK[fmt]
    w = random_blocks(fmt, rows * cols // blk, rows * 7 + cols + len(fmt))
    wd = to_dev(w)
    mv = {"q8_0": K.matvec_q8, "q4k": K.matvec_q4k, "q6k": K.matvec_q6k}[fmt]
    mm = {"q8_0": K.matmul_q8, "q4k": K.matmul_q4k, "q6k": K.matmul_q6k}[fmt]
    for batch in (1, 8, 64):
        xs = acts(orc, fmt, cols, batch, 1000 + batch)
        y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
        if batch == 1:
            mv(y, wd, to_dev(xs), rows, cols)
        else:
            mm(y, wd, to_dev(xs), rows, cols, batch)
        K.sync_check()
        got = y.cpu().numpy()
        ref = orc.matmul(fmt, w, xs, rows, cols, batch)
        if got.tobytes() != ref.tobytes():
            bad = np.argwhere(got.view(np.uint32) != ref.view(np.uint32))
            raise AssertionError(f"{fmt} {rows}x{cols} N={batch}: {len(bad)} values differ, first {bad[:3].tolist()}")


def _same(got, ref, what):
    got = np.ascontiguousarray(got, np.float32)
    ref = np.ascontiguousarray(ref, np.float32)
    if got.tobytes() != ref.tobytes():
        bad = np.flatnonzero(got.view(np.uint32) != ref.view(np.uint32))
        raise AssertionError(f"{what}: {bad.size} of {got.size} differ (first {bad[0]}), "
                             f"max |diff| {float(np.max(np.abs(got.astype(np.float64) - ref))):.3e}")


@pytest.mark.slow
@pytest.mark.parametrize("name", ["llama1b_q8", "llama3b_q4km", "qwen3_4b_q4km", "granite3b_q4km"])
def test_full_size_config_prefill_and_decode(pool, name):
    """Configs 0/2/3/4 at full size: one 64-token prefill chunk, then 8 greedy
    decode steps; every step's logits and sampled KV rows bit-identical to the
    scalar oracle. (Config 0's decode steps hand the SwiGLU output to the down
    projection as Q8_0 blocks quantized by the gate/up kernel.)"""
    import nightrun_b200 as NB
    orc = pool
    orc.set_mode(False)
    cfg = CONFIGS[name]
    gm = NB.Model.synth(cfg, MODEL_SEED)
    blob = orc.synth_nrm(cfg, MODEL_SEED, threads=os.cpu_count() or 8)
    data_off = int.from_bytes(blob[168:176].tobytes(), "little")
    assert gm.data_crc() == orc.crc32(blob[data_off:]), "device model differs from the CPU generator"
    oc = orc.model(blob).ctx(96)
    gc = gm.ctx(96)
    ids = prompt_ids(64, cfg["vocab"])
    _same(gc.prefill_chunk(ids), oc.prefill_chunk(ids), f"{name} 64-token prefill logits")
    tok = gc.next_token
    for step in range(8):
        lo = oc.forward(tok)
        lg = gc.forward(tok)
        _same(lg, lo, f"{name} decode step {step}")
        tok = int(np.argmax(lo))
        assert gc.next_token == tok
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    for layer in (0, 1, cfg["n_layers"] - 1):
        for pos in (0, 63, 71):
            ko, vo = oc.kv(layer, pos, kvd)
            kg, vg = gc.kv(layer, pos)
            assert np.array_equal(ko, kg) and np.array_equal(vo, vg), f"{name} KV layer {layer} pos {pos}"
    gc.close()
    gm.close()


@pytest.mark.slow
def test_attention_past_config3_context(pool):
    """A Qwen3-family model (head_dim 128, q/k norms, NEOX RoPE theta 5e6)
    decoding at positions 2,300..2,315: past config 3's 2,304-position context
    (2,048-token prompt + 256 generated), logits bit-identical to the oracle."""
    import nightrun_b200 as NB
    orc = pool
    orc.set_mode(False)
    cfg = CONFIGS["tiny_qwen3"]
    blob = orc.synth_nrm(cfg, MODEL_SEED)
    oc = orc.model(blob).ctx(2400)
    gc = NB.Model.synth(cfg, MODEL_SEED).ctx(2400)
    ids = prompt_ids(2300, cfg["vocab"])
    _same(gc.prefill(ids), oc.prefill(ids), "2,300-token prefill logits")
    tok = gc.next_token
    for step in range(16):
        lo = oc.forward(tok)
        _same(gc.forward(tok), lo, f"decode at position {2300 + step}")
        tok = int(np.argmax(lo))
    for pos in (0, 1000, 2299, 2315):
        ko, vo = oc.kv(1, pos, cfg["n_kv_heads"] * cfg["head_dim"])
        kg, vg = gc.kv(1, pos)
        assert np.array_equal(ko, kg) and np.array_equal(vo, vg), f"KV pos {pos}"
