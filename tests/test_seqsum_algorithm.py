"""CPU check of the algorithm behind seqsum.cuh's seq_sum_nonneg_warp: the
left-to-right f32 sum of non-negative terms evaluated 256 terms at a time as
integer sums of per-term roundings inside one binade of the running sum (ties
resolved by the running sum's parity), with binade crossings and negative /
non-finite terms added as plain f32 steps. Restated here in Python step for
step as the device code runs it, and compared bit for bit with the plain
sequential chain (vec.rs:4-14, 30-41)."""
import numpy as np
import pytest

F = np.float32
TOP = 1 << 24


def chain(t, init=0.0):
    s = F(init)
    for x in t:
        s = F(s + x)
    return s


def f_bits(x):
    return int(np.array(x, F).view(np.uint32))


def f_from(b):
    return np.array(b & 0xFFFFFFFF, np.uint32).view(F)[()]


def chunked(t, init=0.0, per=8):
    """seq_sum_nonneg_warp step for step: 32 lanes x `per` consecutive terms,
    each lane's increment as a function of the incoming parity, a scan of the
    composed functions, an exact walk for the first crossing / bad term."""
    t = np.asarray(t, F)
    n = len(t)
    i = min(n, 32)
    s = chain(t[:i], init)
    while i < n:
        b = f_bits(s)
        be = b >> 23
        if be < 27 or be > 254:
            s = F(s + t[i])
            i += 1
            continue
        S = (b & 0x7FFFFF) | 0x800000
        scale = f_from((277 - be) << 23)
        lanes = []
        for lane in range(32):
            terms = []
            for k in range(per):
                j = i + lane * per + k
                if j >= n:
                    terms.append(("pad", 0))
                    continue
                x = t[j]
                with np.errstate(over="ignore", invalid="ignore"):
                    T = F(x * scale)
                if not (T < F(16777216.0)) or x < 0:
                    terms.append(("bad", 0))
                    continue
                fl = int(np.trunc(T))
                terms.append(("tie", fl) if F(T - F(fl)) == F(0.5) else ("ok", int(np.rint(T))))
            fn = []
            for p in (0, 1):
                run, acc = p, 0
                for kind, v in terms:
                    if kind == "bad":
                        break
                    d = v + ((run + v) & 1) if kind == "tie" else v
                    acc += d
                    run += d
                fn.append(acc)
            lanes.append((terms, fn))
        excl, tot = [], 0
        for terms, fn in lanes:  # the scan, evaluated at the parity of S
            excl.append(tot)
            tot += fn[(S + tot) & 1]
        event = None
        for lane, (terms, fn) in enumerate(lanes):
            run = S + excl[lane]
            for k, (kind, v) in enumerate(terms):
                if kind == "pad":
                    break
                d = v + ((run + v) & 1) if kind == "tie" else v
                if kind == "bad" or run + d >= TOP:
                    event = (i + lane * per + k, run)
                    break
                run += d
            if event:
                break
        if event is None:
            s = f_from((be << 23) | ((S + tot) & 0x7FFFFF))
            i += 32 * per
            continue
        j, before = event
        s = F(f_from((be << 23) | (before & 0x7FFFFF)) + t[j])
        i = j + 1
    return s


def cases(n, seed):
    g = np.random.default_rng(seed)
    x = g.standard_normal(n).astype(F)
    yield "squares", (x * x).astype(F)
    yield "exps", np.exp(g.standard_normal(n) * 3).astype(F)
    yield "ties", ((g.integers(0, 4, n) * F(0.5)) ** 2).astype(F)
    yield "powers_of_two", np.ldexp(np.ones(n, F), g.integers(-30, 30, n)).astype(F)
    yield "subnormal_squares", ((g.standard_normal(n) * 1e-20).astype(F) ** 2).astype(F)
    h = (x * x).astype(F)
    h[n // 2] = F(9e36)
    yield "one_huge", h
    m = g.standard_normal(n).astype(F)
    m[::3] = np.abs(m[::3])
    yield "mixed_signs", m
    z = np.zeros(n, F)
    z[g.integers(0, n, 3)] = F(1.5)
    yield "mostly_zero", z


@pytest.mark.parametrize("n", [1, 31, 32, 33, 64, 255, 300, 1000, 2048, 4097])
def test_chunked_nonneg_sum_equals_chain(n):
    for name, t in cases(n, n + 11):
        a, b = chain(t), chunked(t)
        assert f_bits(a) == f_bits(b), f"{name} n={n}: chain {a!r} chunked {b!r}"
