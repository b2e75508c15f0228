"""The tolerance mode (NRC_MODE_FAST) of decode steps against the exact
scalar oracle. The north star allows 1e-3 max-abs on the final logits and
requires greedy tokens identical to the reference for the whole generation
of config 0; the mode's sums are trees (block terms, RMSNorm sum of squares,
softmax and V sums) while the per-block integer dots, their roundings and the
activation quantization are the reference's."""
import os

import numpy as np
import pytest

from nightrun_b200.configs import CONFIGS, MODEL_SEED, prompt_ids

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 1e-3  # north star: max-abs on the final logits
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def top2_gap(logits):
    s = np.sort(np.asarray(logits, np.float64))
    return float(s[-1] - s[-2])


@pytest.fixture(scope="module")
def NB():
    import nightrun_b200
    return nightrun_b200


@pytest.mark.parametrize("name", ["tiny_llama_q8", "tiny_llama_q4km", "tiny_qwen3", "tiny_granite"])
def test_fast_decode_within_tolerance(NB, orc, name):
    cfg = CONFIGS[name]
    orc.set_mode(False)
    oc = orc.model(orc.synth_nrm(cfg, MODEL_SEED)).ctx(160)
    gc = NB.Model.synth(cfg, MODEL_SEED).ctx(160)
    gc.set_mode(gc.FAST)
    ids = prompt_ids(24, cfg["vocab"])
    lo = oc.prefill(ids)
    lg = gc.prefill(ids)  # prefill chunks stay exact
    assert lg.tobytes() == lo.tobytes()
    tok = int(np.argmax(lo))
    worst = 0.0
    for step in range(60):
        lo = oc.forward(tok)
        lg = gc.forward(tok)
        worst = max(worst, max_abs(lg, lo))
        assert worst <= LOGIT_ATOL, f"{name} step {step}: max |diff| {worst:.3e}"
        assert gc.next_token == int(np.argmax(lo)), f"{name} step {step}: greedy token differs"
        tok = int(np.argmax(lo))


@pytest.mark.slow
def test_fast_config0_greedy_matches_golden(NB, orc):
    """Config 0 (Llama-3.2-1B architecture, Q8_0): the 128 greedy tokens of the
    fast mode equal the exact scalar oracle's (tests/golden/config0_greedy.npz),
    and the first 24 steps' logits stay within 1e-3 of the oracle's."""
    g = np.load(os.path.join(GOLDEN, "config0_greedy.npz"))
    cfg = CONFIGS["llama1b_q8"]
    m = NB.Model.synth(cfg, int(g["seed"]))
    c = m.ctx(256)
    c.set_mode(c.FAST)
    c.prefill(g["prompt"])
    first = c.next_token
    gen = [first] + [int(t) for t in c.generate(first, len(g["tokens"]) - 1)]
    assert gen == [int(t) for t in g["tokens"]]
    orc.pool_start(os.cpu_count() or 8)
    orc.set_mode(False)
    oc = orc.model(m.export()).ctx(256)
    fc = m.ctx(256)
    fc.set_mode(fc.FAST)
    oc.prefill(g["prompt"])
    fc.prefill(g["prompt"])
    worst, gaps = 0.0, []
    for t in gen[:24]:
        lo = oc.forward(t)
        worst = max(worst, max_abs(fc.forward(t), lo))
        gaps.append(top2_gap(lo))
    print(f"config0 fast: max |logit diff| {worst:.3e} over 24 steps; smallest top-2 gap {min(gaps):.3e}")
    assert worst <= LOGIT_ATOL


@pytest.mark.slow
@pytest.mark.parametrize("name", ["llama3b_q4km", "qwen3_4b_q4km", "granite3b_q4km"])
def test_fast_full_size_configs(NB, orc, name):
    cfg = CONFIGS[name]
    orc.pool_start(os.cpu_count() or 8)
    orc.set_mode(False)
    m = NB.Model.synth(cfg, MODEL_SEED)
    oc = orc.model(orc.synth_nrm(cfg, MODEL_SEED, threads=os.cpu_count() or 8)).ctx(96)
    gc = m.ctx(96)
    gc.set_mode(gc.FAST)
    ids = prompt_ids(64, cfg["vocab"])
    lo = oc.prefill(ids)
    gc.prefill(ids)
    tok = int(np.argmax(lo))
    worst = 0.0
    for step in range(8):
        lo = oc.forward(tok)
        lg = gc.forward(tok)
        worst = max(worst, max_abs(lg, lo))
        assert gc.next_token == int(np.argmax(lo)), f"{name} step {step}"
        tok = int(np.argmax(lo))
    assert worst <= LOGIT_ATOL, f"{name}: max |diff| {worst:.3e}"


@pytest.mark.slow
def test_fast_attention_split_positions(NB, orc):
    """Context of 2,400 positions: the fast attention splits each head's
    positions over 10 CTAs and merges them; decode at 2,300..2,315."""
    cfg = CONFIGS["tiny_qwen3"]
    orc.set_mode(False)
    oc = orc.model(orc.synth_nrm(cfg, MODEL_SEED)).ctx(2400)
    gc = NB.Model.synth(cfg, MODEL_SEED).ctx(2400)
    gc.set_mode(gc.FAST)
    ids = prompt_ids(2300, cfg["vocab"])
    lo = oc.prefill(ids)
    gc.prefill(ids)
    tok = int(np.argmax(lo))
    for step in range(16):
        lo = oc.forward(tok)
        lg = gc.forward(tok)
        assert max_abs(lg, lo) <= LOGIT_ATOL, f"step {step}"
        assert gc.next_token == int(np.argmax(lo))
        tok = int(np.argmax(lo))


def test_mode_switch_keeps_exact_bits(NB, orc):
    """Switching to FAST and back to EXACT: exact steps are bit-identical again."""
    cfg = CONFIGS["tiny_llama_q8"]
    orc.set_mode(False)
    oc = orc.model(orc.synth_nrm(cfg, MODEL_SEED)).ctx(64)
    gc = NB.Model.synth(cfg, MODEL_SEED).ctx(64)
    ids = prompt_ids(8, cfg["vocab"])
    oc.prefill(ids)
    gc.prefill(ids)
    tok = 5
    gc.set_mode(gc.FAST)
    lo = oc.forward(tok)
    assert max_abs(gc.forward(tok), lo) <= LOGIT_ATOL
    gc.set_mode(gc.EXACT)
    for t in (7, 9, 11):
        assert gc.forward(t).tobytes() == oc.forward(t).tobytes()
    with pytest.raises(NB.NrcError):
        gc.set_mode(7)
