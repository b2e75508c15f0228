"""Pins the CPU oracle to the reference's own known-answer tests.

Every test restates one test of crates/nr-tensor/tests/kernels.rs,
crates/nr-tensor/tests/kquant.rs or crates/nr-model/tests/format_malformed.rs
(cited per test) against the C++ restatement in oracle/.
"""
import math

import numpy as np
import pytest

from tests.refdata import Rng, malformed_cases, tiny_nrm
from oracle import oracle as O

F = np.float32


def q8(orc, v):
    return orc.q8_quantize(v)


def q8k(orc, v):
    return orc.quantize_q8k(v)


# ---------------------------------------------------------------- kernels.rs
def test_f16_known_values(orc):  # kernels.rs:43-58
    f = lambda b: float(orc.f16_to_f32(np.array([b], np.uint16))[0])
    assert f(0x3C00) == 1.0
    assert f(0xC000) == -2.0
    assert f(0x3800) == 0.5
    assert f(0x7BFF) == 65504.0
    assert F(f(0x0001)) == F(5.9604645e-8)
    assert f(0x0000) == 0.0
    assert math.isinf(f(0x7C00))
    assert math.isnan(f(0x7E00))
    h = lambda v: int(orc.f32_to_f16(np.array([v], np.float32))[0])
    assert h(1.0) == 0x3C00
    assert h(-2.0) == 0xC000
    assert h(65504.0) == 0x7BFF
    assert h(1e30) == 0x7C00


def test_f16_roundtrip_normals(orc):  # kernels.rs:60-69
    bits = np.arange(0x0400, 0x7C00, dtype=np.uint16)
    for sign in (0, 0x8000):
        b = bits | np.uint16(sign)
        assert np.array_equal(orc.f32_to_f16(orc.f16_to_f32(b)), b)


def test_f16_subnormal_rounds_half_up(orc):  # f16.rs:43-47 (half-up, not RNE)
    # 2^-25 is exactly half of the smallest subnormal: half-up gives 0x0001.
    assert int(orc.f32_to_f16(np.array([2.0 ** -25], np.float32))[0]) == 0x0001
    # 1.5 * 2^-24 sits between 1 and 2 subnormal ulps: half-up gives 0x0002 (RNE would too).
    assert int(orc.f32_to_f16(np.array([1.5 * 2.0 ** -24], np.float32))[0]) == 0x0002
    # 2.5 * 2^-24: RNE would give 2, half-up gives 3.
    assert int(orc.f32_to_f16(np.array([2.5 * 2.0 ** -24], np.float32))[0]) == 0x0003
    # NaN keeps the quiet bit only.
    assert int(orc.f32_to_f16(np.array([np.nan], np.float32))[0]) & 0x7E00 == 0x7E00


def test_quantize_error_bound(orc):  # kernels.rs:71-82
    x = Rng(7).vec(1024)
    blocks = q8(orc, x)
    back = orc.q8_dequantize(blocks)
    scale = orc.f16_to_f32(blocks["d"])
    for i in range(1024):
        assert abs(x[i] - back[i]) <= scale[i // 32] * 0.5 + 1e-6


def test_avx2_matches_scalar_q8(orc):  # kernels.rs:84-100
    rng = Rng(42)
    for blocks in [1, 3, 64, 65]:
        w = q8(orc, rng.vec(blocks * 32))
        x = q8(orc, rng.vec(blocks * 32))
        s = orc.dot("q8_0", w, x, 0)
        v = orc.dot("q8_0", w, x, 1)
        tol = 1e-5 * max(float(blocks), 1.0) + 1e-6
        assert abs(s - v) <= tol * max(abs(s), 1.0)


def test_matvec_matches_f32_reference(orc):  # kernels.rs:102-128
    rng = Rng(1234)
    rows, cols = 48, 128
    wf = rng.vec(rows * cols)
    xf = rng.vec(cols)
    w, x = q8(orc, wf), q8(orc, xf)
    y = orc.matvec("q8_0", w, x, rows, cols)
    wd = orc.q8_dequantize(w).reshape(rows, cols)
    xd = orc.q8_dequantize(x)
    for r in range(rows):
        expect = F(0)
        for a, b in zip(wd[r], xd):
            expect = F(expect + F(a * b))
        assert abs(y[r] - expect) <= 1e-4 * max(abs(expect), 1.0)


def test_rmsnorm_reference(orc):  # kernels.rs:130-142
    x = np.array([1, 2, 3, 4], np.float32)
    w = np.array([0.5, 1.0, 1.5, 2.0], np.float32)
    out = orc.rmsnorm(x, w, 1e-5)
    ms = float(np.sum(x * x)) / 4
    scale = 1.0 / math.sqrt(ms + 1e-5)
    for i in range(4):
        assert abs(out[i] - x[i] * scale * w[i]) < 1e-6


def test_softmax_reference(orc):  # kernels.rs:144-154
    x = orc.softmax([0.0, 1.0, 2.0])
    e = [1.0, math.exp(1.0), math.exp(2.0)]
    for i in range(3):
        assert abs(x[i] - e[i] / sum(e)) < 1e-6
    assert abs(float(np.sum(x)) - 1.0) < 1e-6


def test_swiglu_reference(orc):  # kernels.rs:156-165
    g = orc.swiglu([1.0, -1.0], [2.0, 3.0])
    assert abs(g[0] - 1.0 / (1.0 + math.exp(-1.0)) * 2.0) < 1e-6
    assert abs(g[1] - (-1.0 / (1.0 + math.exp(1.0))) * 3.0) < 1e-6


def test_rope_identity_at_pos0(orc):  # kernels.rs:167-176
    freqs = orc.rope_freqs(64, 500000.0)
    orig = Rng(5).vec(64)
    x = orc.rope_apply(orig, 64, freqs, 0, 0)
    assert np.array_equal(x, orig)


def test_rope_rotation_matches_trig(orc):  # kernels.rs:178-197
    hd = 8
    freqs = orc.rope_freqs(hd, 10000.0)
    assert abs(freqs[0] - 1.0) < 1e-6
    orig = np.arange(1, hd + 1, dtype=np.float32)
    x = orc.rope_apply(orig, hd, freqs, 3, 0)
    for i in range(hd // 2):
        ang = 3 * float(freqs[i])
        a, b = float(orig[2 * i]), float(orig[2 * i + 1])
        assert abs(x[2 * i] - (a * math.cos(ang) - b * math.sin(ang))) < 1e-4
        assert abs(x[2 * i + 1] - (a * math.sin(ang) + b * math.cos(ang))) < 1e-4


def test_rope_llama3_scaling_behaviour(orc):  # kernels.rs:199-226
    hd = 64
    plain = orc.rope_freqs(hd, 500000.0)
    scaled = orc.rope_freqs(hd, 500000.0, (32.0, 1.0, 4.0, 8192.0))
    assert plain[0] == scaled[0]
    last = hd // 2 - 1
    assert 2 * math.pi / plain[last] > 8192.0
    assert abs(scaled[last] - plain[last] / 32.0) < plain[last] * 1e-5
    assert np.all(scaled[1:] < scaled[:-1])


def test_argmax_works(orc):  # kernels.rs:228-231
    assert orc.argmax([0.1, 4.0, -2.0, 4.0]) == 1


@pytest.mark.parametrize("fast", [False, True])
def test_matmul_q8_bit_equals_matvec(orc, fast):  # kernels.rs:277-292
    orc.set_mode(fast)
    try:
        rng = Rng(202)
        rows, cols, batch = 48, 256, 4
        w = q8(orc, rng.vec(rows * cols))
        xs = q8(orc, rng.vec(batch * cols))
        bpr = cols // 32
        ym = orc.matmul("q8_0", w, xs, rows, cols, batch)
        for b in range(batch):
            yv = orc.matvec("q8_0", w, xs[b * bpr:(b + 1) * bpr].copy(), rows, cols)
            assert np.array_equal(ym[b], yv)
    finally:
        orc.set_mode(False)


# ----------------------------------------------------------------- kquant.rs
def test_q8k_quantization_properties(orc):  # kquant.rs:54-76
    rng = Rng(11)
    for src in [rng.vec(512), rng.adversarial(512)]:
        blocks = q8k(orc, src)
        for bi, b in enumerate(blocks):
            qs = b["qs"].astype(np.int32)
            for g in range(16):
                assert qs[g * 16:(g + 1) * 16].sum() == int(b["bsums"][g])
            chunk = src[bi * 256:(bi + 1) * 256]
            back = qs.astype(np.float32) * b["d"]
            assert np.all(np.abs(back - chunk) <= abs(b["d"]) * 0.5 + 1e-6)


def test_q4k_dequant_roundtrip(orc):  # kquant.rs:78-101
    rng = Rng(21)
    for src in [rng.vec(256), rng.adversarial(256)]:
        block = orc.quantize_q4k_ref(src)
        back = orc.dequant_q4k(block)
        d = float(orc.f16_to_f32(block["d"])[0])
        sc = block["scales"][0]
        for j in range(8):
            s = (sc[j] & 63) if j < 4 else ((sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4))
            step = d * float(s)
            for k in range(32):
                i = j * 32 + k
                tol = step * 0.75 + max(step, 1e-3)
                assert abs(back[i] - src[i]) <= tol


def test_q6k_dequant_roundtrip(orc):  # kquant.rs:103-136 (zero tolerance on packing)
    rng = Rng(31)
    for src in [rng.vec(256), rng.adversarial(256)]:
        block = orc.quantize_q6k_ref(src)
        d = orc.f16_to_f32(block["d"])[0]
        back = orc.dequant_q6k(block)
        for i in range(256):
            sc = F(d * F(int(block["scales"][0][i // 16])))
            if sc != 0:
                r = F(src[i] / sc)
                r = int(F(r + F(0.5))) if r >= 0 else int(F(r - F(0.5)))
                q = min(max(r + 32, 0), 63) - 32
            else:
                q = 0
            expect = F(sc * F(q))
            assert abs(back[i] - expect) <= abs(expect) * 1e-6 + 1e-7


def _dequant_ref_dot(orc, w, x, fmt):
    deq = orc.dequant_q4k if fmt == "q4k" else orc.dequant_q6k
    expect = 0.0
    for bw, bx in zip(w, x):
        wd = deq(np.array([bw]))
        xd = bx["qs"].astype(np.float32) * bx["d"]
        expect += float(np.sum(wd.astype(np.float64) * xd.astype(np.float64)))
    return expect


@pytest.mark.parametrize("fmt,seed", [("q4k", 41), ("q6k", 51)])
def test_kquant_dot_matches_dequant_reference(orc, fmt, seed):  # kquant.rs:138-166, 269-295
    rng = Rng(seed)
    quant = orc.quantize_q4k_ref if fmt == "q4k" else orc.quantize_q6k_ref
    for blocks in [1, 3, 10]:
        w = quant(rng.adversarial(blocks * 256))
        x = q8k(orc, rng.vec(blocks * 256))
        got = orc.dot(fmt, w, x, 0)
        expect = _dequant_ref_dot(orc, w, x, fmt)
        assert abs(got - expect) <= 1e-3 * max(abs(expect), 1.0)


@pytest.mark.parametrize("fmt,seed", [("q4k", 61), ("q6k", 71)])
def test_avx2_matches_scalar_kquant(orc, fmt, seed):  # kquant.rs:168-208
    rng = Rng(seed)
    quant = orc.quantize_q4k_ref if fmt == "q4k" else orc.quantize_q6k_ref
    for blocks in [1, 5, 16]:
        w = quant(rng.adversarial(blocks * 256))
        x = q8k(orc, rng.vec(blocks * 256))
        s, v = orc.dot(fmt, w, x, 0), orc.dot(fmt, w, x, 1)
        assert abs(s - v) <= 1e-4 * max(abs(s), 1.0)


def saturated_blocks(orc):
    """Blocks of kquant.rs:213-228: all-max Q4_K scales/mins/quants, extreme Q6_K."""
    q4 = np.zeros(1, O.Q4K)
    q4["d"] = orc.f32_to_f16(np.array([0.9], np.float32))
    q4["dmin"] = orc.f32_to_f16(np.array([1.7], np.float32))
    q4["scales"] = 0xFF
    q4["qs"] = 0xFF
    q6 = np.zeros(1, O.Q6K)
    q6["ql"] = 0xFF
    q6["qh"] = 0xFF
    q6["scales"] = -128
    q6["d"] = orc.f32_to_f16(np.array([1.3], np.float32))
    return q4, q6


def test_avx2_matches_scalar_saturated_blocks(orc):  # kquant.rs:210-245
    q4, q6 = saturated_blocks(orc)
    x = q8k(orc, Rng(81).adversarial(256))
    s4, v4 = orc.dot("q4k", q4, x, 0), orc.dot("q4k", q4, x, 1)
    assert abs(s4 - v4) <= 1e-4 * max(abs(s4), 1.0)
    s6, v6 = orc.dot("q6k", q6, x, 0), orc.dot("q6k", q6, x, 1)
    assert abs(s6 - v6) <= 1e-4 * max(abs(s6), 1.0)


def test_matvec_kquant_matches_dot(orc):  # kquant.rs:247-267
    rng = Rng(91)
    rows, cols = 48, 512
    w4 = orc.quantize_q4k_ref(rng.vec(rows * cols))
    x = q8k(orc, rng.vec(cols))
    y = orc.matvec("q4k", w4, x, rows, cols)
    bpr = cols // 256
    for r in range(rows):
        expect = orc.dot("q4k", w4[r * bpr:(r + 1) * bpr].copy(), x, 0)
        assert abs(y[r] - expect) <= 1e-4 * max(abs(expect), 1.0)


@pytest.mark.parametrize("fast", [False, True])
def test_kquant_matmul_bit_equals_matvec(orc, fast):  # kquant.rs:297-329
    orc.set_mode(fast)
    try:
        rng = Rng(101)
        rows, cols, batch = 32, 512, 5
        w4 = orc.quantize_q4k_ref(rng.vec(rows * cols))
        w6 = orc.quantize_q6k_ref(rng.vec(rows * cols))
        xs = q8k(orc, rng.vec(batch * cols))
        bpr = cols // 256
        ym4 = orc.matmul("q4k", w4, xs, rows, cols, batch)
        ym6 = orc.matmul("q6k", w6, xs, rows, cols, batch)
        for b in range(batch):
            x = xs[b * bpr:(b + 1) * bpr].copy()
            assert np.array_equal(ym4[b], orc.matvec("q4k", w4, x, rows, cols))
            assert np.array_equal(ym6[b], orc.matvec("q6k", w6, x, rows, cols))
    finally:
        orc.set_mode(False)


# ------------------------------------------------------ format_malformed.rs
def test_valid_tiny_file_parses(orc):  # format_malformed.rs:100-108
    m = orc.model(np.frombuffer(bytes(tiny_nrm()), np.uint8))
    assert m.meta.dim == 8
    t = m.tensors()
    assert (t[0][5], t[0][6]) == (8, 8)
    assert m.verify()


@pytest.mark.parametrize("name,blob,meta_crc", malformed_cases(), ids=[c[0] for c in malformed_cases()])
def test_malformed_rejects(orc, name, blob, meta_crc):  # format_malformed.rs:110-206
    with pytest.raises(ValueError) as e:
        orc.model(np.frombuffer(blob, np.uint8))
    if meta_crc:
        assert "MetaCrc" in str(e.value)


def test_crc32_known_vector(orc):  # crc32.rs (IEEE CRC-32 check value)
    assert orc.crc32(b"123456789") == 0xCBF43926
    data = np.random.default_rng(0).integers(0, 256, 10007, dtype=np.uint8)
    import zlib
    assert orc.crc32(data) == zlib.crc32(data.tobytes())
