"""Several sequences decoded together (nrc_batch_*): each sequence's logits,
greedy tokens and KV cache must be bit-identical to an independent
single-sequence run of the scalar oracle (crates/nr-model/src/infer.rs:
510-778 per sequence), whatever the other sequences in the pass are doing:
ragged prompt lengths, prompts split across passes, several sequences per
pass, then batched decode steps at different positions."""
import os

import numpy as np
import pytest

from nightrun_b200.configs import CONFIGS, MODEL_SEED, prompt_ids

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def NB():
    import nightrun_b200
    return nightrun_b200


def prompts_for(cfg, lens):
    return [prompt_ids(n, cfg["vocab"], seed=MODEL_SEED + 11 + i) for i, n in enumerate(lens)]


def run_oracle(orc, blob, prompts, steps, ctx):
    """Independent scalar contexts: prefill logits' choice, then `steps` greedy
    steps with their logits."""
    orc.set_mode(False)
    out = []
    for pr in prompts:
        c = orc.model(blob).ctx(ctx)
        tok = int(np.argmax(c.prefill(pr)))
        toks, logits = [tok], []
        for _ in range(steps):
            lo = c.forward(toks[-1])
            logits.append(lo)
            toks.append(int(np.argmax(lo)))
        out.append((toks, logits, c))
    return out


@pytest.mark.parametrize("name,lens", [
    ("tiny_llama_q8", [3, 17, 64, 70, 1]),
    ("tiny_llama_q4km", [40, 2, 33]),
    ("tiny_qwen3", [9, 9, 9, 9, 9, 9, 9, 9, 9]),
    ("tiny_granite", [65, 1, 128, 5]),
])
def test_batch_matches_independent_sequences(NB, orc, name, lens):
    cfg = CONFIGS[name]
    blob = orc.synth_nrm(cfg, MODEL_SEED)
    prompts = prompts_for(cfg, lens)
    steps = 12
    ref = run_oracle(orc, blob, prompts, steps, 200)
    b = NB.Model.synth(cfg, MODEL_SEED).batch(200, len(lens))
    nxt = b.prefill(prompts)
    assert [int(t) for t in nxt] == [r[0][0] for r in ref]
    for q, n in enumerate(lens):
        assert b.pos(q) == n
    for i in range(steps):
        lg, nxt = b.step()
        for q in range(len(lens)):
            assert lg[q].tobytes() == ref[q][1][i].tobytes(), f"{name} seq {q} step {i}"
            assert int(nxt[q]) == ref[q][0][i + 1]
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    for q, n in enumerate(lens):
        for pos in (0, n - 1, n + steps - 1):
            ko, vo = ref[q][2].kv(cfg["n_layers"] - 1, pos, kvd)
            kg, vg = b.kv(q, cfg["n_layers"] - 1, pos)
            assert np.array_equal(ko, kg) and np.array_equal(vo, vg), f"{name} seq {q} pos {pos} KV"
    # Device-side generation continues every sequence exactly like the oracle.
    more = b.generate(6)
    for q in range(len(lens)):
        c = ref[q][2]
        t = ref[q][0][-1]
        want = []
        for _ in range(6):
            t = int(np.argmax(c.forward(t)))
            want.append(t)
        assert [int(x) for x in more[q]] == want, f"{name} seq {q} generate"


def test_batch_errors(NB):
    cfg = CONFIGS["tiny_llama_q8"]
    m = NB.Model.synth(cfg, MODEL_SEED)
    b = m.batch(16, 3)
    with pytest.raises(NB.NrcError) as e:
        b.step()  # no prompt yet
    assert e.value.name == "INVALID"
    with pytest.raises(NB.NrcError) as e:
        b.prefill([[1, 2], [], [3]])
    assert e.value.name == "BAD_BATCH"
    with pytest.raises(NB.NrcError) as e:
        b.prefill([[1] * 17, [2], [3]])
    assert e.value.name == "CTX_FULL"
    b.prefill([[1] * 15, [2], [3]])
    with pytest.raises(NB.NrcError) as e:
        b.generate(2)  # sequence 0 would pass position 16
    assert e.value.name == "CTX_FULL"
    b.step()
    # The single-sequence entry points refuse a multi-sequence context.
    with pytest.raises(NB.NrcError) as e:
        NB._lib.check(NB.lib().nrc_ctx_forward(b.h, 1, None, None))
    assert e.value.name == "INVALID"
    b.reset()
    assert b.pos(0) == 0


@pytest.mark.slow
def test_config4_batched_decode_full_size(NB, orc):
    """Config 4 (Granite-4.1-3B architecture, Q4_K/Q6_K mix, muP scalars) at
    full size: 16 sequences with ragged prompts decoded together, every logit
    of 3 decode steps bit-identical to 16 independent scalar contexts."""
    cfg = CONFIGS["granite3b_q4km"]
    orc.pool_start(os.cpu_count() or 8)
    blob = orc.synth_nrm(cfg, MODEL_SEED, threads=os.cpu_count() or 8)
    lens = [4 + q for q in range(16)]
    prompts = prompts_for(cfg, lens)
    steps = 3
    ref = run_oracle(orc, blob, prompts, steps, 64)
    b = NB.Model.synth(cfg, MODEL_SEED).batch(64, 16)
    nxt = b.prefill(prompts)
    assert [int(t) for t in nxt] == [r[0][0] for r in ref]
    for i in range(steps):
        lg, nxt = b.step()
        for q in range(16):
            assert lg[q].tobytes() == ref[q][1][i].tobytes(), f"seq {q} step {i}"
