"""The oracle's expf (the function vec.rs:34,47 and sample.rs:70 call) is the
correctly rounded binary32 exp: checked here on a strided sample of every
binary32 input against float64 exp (disagreements settled with 60-digit
decimal arithmetic), and its all-input chunk hashes against the committed
tests/golden/expf_cr_hashes.bin that the GPU test uses. The full 2^32-input
check against long-double expl is oracle/check_expf.cpp."""
import os
from decimal import Decimal, getcontext

import numpy as np

GOLD = os.path.join(os.path.dirname(__file__), "golden", "expf_cr_hashes.bin")


def exact_round_exp(x):
    getcontext().prec = 60
    e = Decimal(float(x)).exp()
    lo = np.float32(float(e))
    # Pick the float32 nearest to e (ties to even) among lo's neighbours.
    cands = [np.nextafter(lo, np.float32(-np.inf)), lo, np.nextafter(lo, np.float32(np.inf))]
    best = min(cands, key=lambda c: (abs(Decimal(float(c)) - e), int(np.float32(c).view(np.uint32)) & 1))
    return np.float32(best)


def test_expf_sampled_inputs_correctly_rounded(orc):
    bits = np.arange(0, 1 << 32, 509, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    y = orc.expf(x)
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        ref = np.exp(x.astype(np.float64)).astype(np.float32)
    nan = np.isnan(x)
    assert np.all(np.isnan(y[nan]))
    diff = np.flatnonzero((y.view(np.uint32) != ref.view(np.uint32)) & ~nan)
    for i in diff:  # float64 double rounding: settle with decimal arithmetic
        assert y[i] == exact_round_exp(x[i]), f"x={x[i]!r}: {y[i]!r}"
    assert diff.size < 50


def test_expf_chunk_hashes_match_golden(orc):
    gold = np.fromfile(GOLD, np.uint64)
    assert gold.size == 4096
    for c in (0, 1, 1000, 2047, 2048, 2100, 3071, 3200, 4095):
        assert orc.expf_hash(c, 1)[0] == gold[c], f"chunk {c}"


def test_expf_edges(orc):
    x = np.array([0.0, -0.0, np.inf, -np.inf, 88.72283, 88.72284, -103.97208, -103.97209, -200.0], np.float32)
    y = orc.expf(x)
    assert y[0] == 1.0 and y[1] == 1.0 and y[2] == np.inf and y[3] == 0.0
    assert np.isfinite(y[4]) and y[5] == np.inf
    assert y[6] > 0.0 and y[8] == 0.0
