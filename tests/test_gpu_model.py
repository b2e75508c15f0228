"""GPU parity of the model-level C ABI (synthetic models, forward, prefill,
greedy decode) against the CPU oracle's scalar path and committed fixtures.

Tolerances (north star): final logits within max-abs 1e-3 of the scalar
reference; greedy tokens identical. Prefill must be bit-identical to
token-by-token decode on the GPU, logits and KV cache
(crates/nr-model/tests/prefill.rs:45-70, 91-133).
"""
import os

import numpy as np
import pytest

from nightrun_b200.configs import CONFIGS, MODEL_SEED, prompt_ids

pytestmark = pytest.mark.gpu

TINY = ["tiny_llama_q8", "tiny_llama_q4km", "tiny_qwen3", "tiny_granite"]
LOGIT_ATOL = 1e-3
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


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
    worst = 0.0
    for t in ids:
        lo = oc.forward(t)
        lg = gc.forward(t)
        worst = max(worst, float(np.max(np.abs(lo - lg))))
        assert int(np.argmax(lg)) == int(np.argmax(lo)) or np.sort(lo)[-1] - np.sort(lo)[-2] < 1e-4
    assert worst <= LOGIT_ATOL, f"{name}: max |logit diff| {worst}"
    # The f16 KV cache agrees to within an f16 ulp step of the same values.
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    for layer in range(cfg["n_layers"]):
        for pos in (0, 17, 39):
            ko, vo = oc.kv(layer, pos, kvd)
            kg, vg = gc.kv(layer, pos, kvd)
            assert np.max(np.abs(orc.f16_to_f32(ko) - orc.f16_to_f32(kg))) <= 1e-2
            assert np.max(np.abs(orc.f16_to_f32(vo) - orc.f16_to_f32(vg))) <= 1e-2


@pytest.mark.parametrize("name", TINY)
def test_prefill_bit_identical_to_sequential(NB, name):  # prefill.rs:91-133 lengths (<= 129)
    cfg = CONFIGS[name]
    m = NB.Model.synth(cfg, MODEL_SEED)
    seq, bat = m.ctx(320), m.ctx(320)
    ids = prompt_ids(140, cfg["vocab"])
    for n in (1, 7, 15, 17, 31, 33, 63, 65, 127, 128, 129):
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
    assert float(np.max(np.abs(lg - g["logits_prefill"]))) <= LOGIT_ATOL
    first = c.next_token
    gen = [first] + [int(t) for t in c.generate(first, len(g["tokens"]) - 1)]
    assert gen == [int(t) for t in g["tokens"]]
