"""GPU parity of the model-level C ABI (synthetic models, forward, prefill,
greedy decode) against the CPU oracle's scalar path and committed fixtures.

The device path reproduces the reference's scalar kernels operation by
operation (integer block dots, the same f32 roundings in the same order,
correctly rounded expf), so logits and the f16 KV cache are compared BIT FOR
BIT with the scalar oracle; the north star's max-abs 1e-3 on final logits is
reported alongside as a diagnostic when bits differ. Prefill must be
bit-identical to token-by-token decode, logits and KV cache
(crates/nr-model/tests/prefill.rs:45-70, 91-133).
"""
import os

import numpy as np
import pytest

from nightrun_b200.configs import CONFIGS, MODEL_SEED, prompt_ids

pytestmark = pytest.mark.gpu

TINY = ["tiny_llama_q8", "tiny_llama_q4km", "tiny_qwen3", "tiny_granite"]
LOGIT_ATOL = 1e-3  # north-star tolerance, reported when bits differ
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def assert_same_bits(got, ref, what):
    got = np.ascontiguousarray(got, np.float32)
    ref = np.ascontiguousarray(ref, np.float32)
    assert got.shape == ref.shape, what
    if got.tobytes() != ref.tobytes():
        bad = np.flatnonzero(got.view(np.uint32) != ref.view(np.uint32))
        diff = float(np.max(np.abs(got.astype(np.float64) - ref)))
        raise AssertionError(f"{what}: {bad.size} of {got.size} values differ (first at {bad[0]}), "
                             f"max |diff| {diff:.3e} (north-star tolerance {LOGIT_ATOL})")


@pytest.fixture(scope="module")
def NB():
    import nightrun_b200
    return nightrun_b200


_blobs = {}


def oracle_blob(orc, name, seed=MODEL_SEED):
    key = (name, seed)
    if key not in _blobs:
        _blobs[key] = orc.synth_nrm(CONFIGS[name], seed)
    return _blobs[key]


@pytest.mark.parametrize("name", TINY)
def test_synth_model_bytes_match_cpu_generator(NB, orc, name):
    m = NB.Model.synth(CONFIGS[name], MODEL_SEED)
    blob = m.export()
    ref = oracle_blob(orc, name)
    assert blob.size == ref.size
    assert blob.tobytes() == ref.tobytes()


@pytest.mark.parametrize("name", ["tiny_llama_q8", "tiny_qwen3"])
def test_load_upload_roundtrip(NB, orc, name):
    ref = oracle_blob(orc, name)
    m = NB.Model.load(ref, verify_crc=True)
    assert m.data_crc() == orc.crc32(ref[int.from_bytes(ref[168:176].tobytes(), "little"):])
    assert m.export().tobytes() == ref.tobytes()
    bad = ref.copy()
    bad[-1] ^= 0xFF
    with pytest.raises(NB.NrcError) as e:
        NB.Model.load(bad, verify_crc=True)
    assert e.value.name == "DATA_CRC"


@pytest.mark.parametrize("name", TINY)
def test_forward_matches_oracle(NB, orc, name):
    cfg = CONFIGS[name]
    orc.set_mode(False)
    om = orc.model(oracle_blob(orc, name))
    oc = om.ctx(160)
    gm = NB.Model.synth(cfg, MODEL_SEED)
    gc = gm.ctx(160)
    ids = prompt_ids(40, cfg["vocab"])
    for i, t in enumerate(ids):
        assert_same_bits(gc.forward(t), oc.forward(t), f"{name} step {i} logits")
    # The f16 KV cache holds identical bits.
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    for layer in range(cfg["n_layers"]):
        for pos in (0, 17, 39):
            ko, vo = oc.kv(layer, pos, kvd)
            kg, vg = gc.kv(layer, pos)
            assert np.array_equal(ko, kg), f"{name} layer {layer} pos {pos} K cache"
            assert np.array_equal(vo, vg), f"{name} layer {layer} pos {pos} V cache"


@pytest.mark.parametrize("name", ["tiny_llama_q8", "tiny_granite"])
def test_prefill_matches_oracle_prefill(NB, orc, name):
    """Batched prefill (tensor-core GEMM for Q8_0 chunks > 8 tokens) against the
    oracle's prefill (infer.rs:601-750) over ragged chunk lengths."""
    cfg = CONFIGS[name]
    orc.set_mode(False)
    oc = orc.model(oracle_blob(orc, name)).ctx(256)
    gc = NB.Model.synth(cfg, MODEL_SEED).ctx(256)
    ids = prompt_ids(200, cfg["vocab"])
    p = 0
    for n in (9, 64, 17, 1, 33, 40):
        assert_same_bits(gc.prefill(ids[p:p + n]), oc.prefill(ids[p:p + n]), f"{name} chunk at {p}+{n}")
        p += n


@pytest.mark.parametrize("name", TINY)
def test_prefill_bit_identical_to_sequential(NB, name):  # all 16 lengths of prefill.rs:91-133
    cfg = CONFIGS[name]
    m = NB.Model.synth(cfg, MODEL_SEED)
    seq, bat = m.ctx(520), m.ctx(520)
    ids = prompt_ids(520, cfg["vocab"])
    for n in (1, 7, 15, 17, 31, 33, 63, 65, 127, 128, 129, 255, 257, 511, 512, 513):
        seq.reset()
        bat.reset()
        ls = None
        for t in ids[:n]:
            ls = seq.forward(t)
        lb = bat.prefill(ids[:n])
        assert seq.pos == bat.pos == n
        assert ls.tobytes() == lb.tobytes(), f"len {n}: prefill logits differ"
        # Identical KV cache: the next decode step matches bit for bit.
        nxt = int(np.argmax(ls))
        assert seq.forward(nxt).tobytes() == bat.forward(nxt).tobytes(), f"len {n}: post-prefill step differs"


@pytest.mark.parametrize("name", TINY)
def test_greedy_generation_matches_oracle(NB, orc, name):
    cfg = CONFIGS[name]
    orc.set_mode(False)
    oc = orc.model(oracle_blob(orc, name)).ctx(200)
    ids = prompt_ids(24, cfg["vocab"])
    lo = oc.prefill(ids)
    ref = []
    nxt = int(np.argmax(lo))
    for _ in range(48):
        ref.append(nxt)
        nxt = int(np.argmax(oc.forward(nxt)))
    gm = NB.Model.synth(cfg, MODEL_SEED)
    gc = gm.ctx(200)
    lg = gc.prefill(ids)
    first = gc.next_token
    assert first == int(np.argmax(lg)) == ref[0]
    gen = gc.generate(first, 47)
    got = [first] + [int(t) for t in gen]
    assert got == ref
    # Device-loop generation equals host-driven greedy decode.
    gc2 = gm.ctx(200)
    gc2.prefill(ids)
    host = [gc2.next_token]
    for _ in range(47):
        host.append(gc2.forward_greedy(host[-1]))
    assert host == got


def test_context_limits_and_errors(NB):
    cfg = CONFIGS["tiny_llama_q8"]
    m = NB.Model.synth(cfg, MODEL_SEED)
    c = m.ctx(8)
    with pytest.raises(NB.NrcError) as e:
        c.prefill_chunk(list(range(65)))
    assert e.value.name == "BAD_BATCH"
    with pytest.raises(NB.NrcError) as e:
        c.forward(cfg["vocab"])
    assert e.value.name == "BAD_TOKEN"
    c.prefill(list(range(8)))
    assert c.remaining() == 0
    with pytest.raises(NB.NrcError) as e:
        c.forward(1)
    assert e.value.name == "CTX_FULL"
    c.reset()
    assert c.pos == 0 and c.remaining() == 8


def test_context_limit_counts_enqueued_steps(NB):
    """Decode steps enqueued with decode_async but not yet synced count against
    the context window: every entry point rejects on the host (CTX_FULL) before
    any kernel could append a KV row past the end (infer.rs:513, 605)."""
    cfg = CONFIGS["tiny_llama_q8"]
    m = NB.Model.synth(cfg, MODEL_SEED)
    c = m.ctx(12)
    c.prefill(list(range(4)))
    c.decode_async(5)  # device position reaches 9 once these run
    assert c.remaining() == 3
    for call in (lambda: c.decode_async(4), lambda: c.prefill_chunk([1, 2, 3, 4]),
                 lambda: c.prefill([1, 2, 3, 4]), lambda: c.generate(1, 4)):
        with pytest.raises(NB.NrcError) as e:
            call()
        assert e.value.name == "CTX_FULL"
    c.decode_async(3)
    with pytest.raises(NB.NrcError) as e:
        c.forward(1)
    assert e.value.name == "CTX_FULL"
    c.sync()
    assert c.pos == 12 and c.remaining() == 0
    # The same steps synced one call at a time give the same tokens.
    c2 = m.ctx(12)
    c2.prefill(list(range(4)))
    toks = [c2.next_token]
    for _ in range(8):
        toks.append(c2.forward_greedy(toks[-1]))
    c.reset()
    c.prefill(list(range(4)))
    c.decode_async(8)
    assert c.sync() == toks[-1]


@pytest.mark.slow
def test_config0_greedy_matches_golden(NB):
    """Config 0 (Llama-3.2-1B architecture, Q8_0): 64-token prompt, 128 greedy tokens,
    against the scalar oracle's tokens committed in tests/golden/config0_greedy.npz."""
    g = np.load(os.path.join(GOLDEN, "config0_greedy.npz"))
    cfg = CONFIGS["llama1b_q8"]
    m = NB.Model.synth(cfg, int(g["seed"]))
    assert m.data_crc() == int(g["data_crc"])
    c = m.ctx(256)
    lg = c.prefill(g["prompt"])
    assert_same_bits(lg, g["logits_prefill"], "config 0 prefill logits")
    first = c.next_token
    gen = [first] + [int(t) for t in c.generate(first, len(g["tokens"]) - 1)]
    assert gen == [int(t) for t in g["tokens"]]
