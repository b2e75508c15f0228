"""GPU parity of the kernel-level C ABI against the CPU oracle.

Integer / byte work (quantizers, f16 conversion, dequantization) and the
matvec/matmul outputs must be bit-identical to the reference's scalar code
(the GEMV and the tensor-core GEMM keep the scalar summation order);
rmsnorm/softmax/swiglu keep the reference's sequential sums and a correctly
rounded expf, so they are bit-identical too (stricter than the reference's own
1e-6 relative tolerance, crates/nr-tensor/tests/kernels.rs:130-165).
"""
import os

import numpy as np
import pytest
import torch

from tests.refdata import Rng
from oracle import oracle as O

pytestmark = pytest.mark.gpu

F = np.float32


@pytest.fixture(scope="module")
def K():
    from nightrun_b200 import kernels
    return kernels


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def blocks_dev(b):
    return dev(np.frombuffer(b.tobytes(), np.uint8).copy())


def host_bytes(t):
    torch.cuda.synchronize()
    return t.cpu().numpy().tobytes()


def rand_bits_f32(n, seed):
    r = np.random.default_rng(seed)
    x = r.standard_normal(n).astype(np.float32) * r.choice([1e-6, 1e-3, 1.0, 30.0, 1e4], n).astype(np.float32)
    return x


def test_f16_to_f32_all_patterns(K, orc):
    bits = np.arange(65536, dtype=np.uint16)
    out = torch.empty(65536, dtype=torch.float32, device="cuda")
    K.f16_to_f32(dev(bits.view(np.int16)), out)
    assert host_bytes(out) == orc.f16_to_f32(bits).tobytes()


def test_f32_to_f16_matches_reference(K, orc):
    r = np.random.default_rng(3)
    vals = np.concatenate([
        r.integers(0, 2 ** 32, 200000, dtype=np.uint64).astype(np.uint32).view(np.float32),
        rand_bits_f32(100000, 4),
        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 65504.0, 65520.0, 1e30, 2.0 ** -25, 1.5 * 2.0 ** -24,
                  2.5 * 2.0 ** -24, 6e-8, -6e-8, 2.0 ** -14, 2.0 ** -15], np.float32)])
    out = torch.empty(vals.size, dtype=torch.int16, device="cuda")
    K.f32_to_f16(dev(vals), out)
    assert host_bytes(out) == orc.f32_to_f16(vals).tobytes()


@pytest.mark.parametrize("gen", ["vec", "adversarial", "zeros"])
def test_quantize_q8_0_bytes(K, orc, gen):
    rng = Rng(7)
    x = {"vec": lambda: rng.vec(4096), "adversarial": lambda: rng.adversarial(4096),
         "zeros": lambda: np.zeros(4096, np.float32)}[gen]()
    out = torch.empty(4096 // 32 * 34, dtype=torch.uint8, device="cuda")
    K.quantize(dev(x), out)
    assert host_bytes(out) == orc.q8_quantize(x).tobytes()
    back = torch.empty(4096, dtype=torch.float32, device="cuda")
    K.dequantize(out, back)
    assert host_bytes(back) == orc.q8_dequantize(orc.q8_quantize(x)).tobytes()


@pytest.mark.parametrize("gen", ["vec", "adversarial", "zeros"])
def test_quantize_q8k_bytes(K, orc, gen):
    rng = Rng(11)
    x = {"vec": lambda: rng.vec(2048), "adversarial": lambda: rng.adversarial(2048),
         "zeros": lambda: np.zeros(2048, np.float32)}[gen]()
    out = torch.empty(2048 // 256 * 292, dtype=torch.uint8, device="cuda")
    K.quantize_q8k(dev(x), out)
    assert host_bytes(out) == orc.quantize_q8k(x).tobytes()


@pytest.mark.parametrize("fmt", ["q4k", "q6k"])
def test_dequant_kquant_bit_exact(K, orc, fmt):
    rng = Rng(21)
    src = np.concatenate([rng.vec(256 * 8), rng.adversarial(256 * 8)])
    b = orc.quantize_q4k_ref(src) if fmt == "q4k" else orc.quantize_q6k_ref(src)
    out = torch.empty(src.size, dtype=torch.float32, device="cuda")
    (K.dequant_q4k if fmt == "q4k" else K.dequant_q6k)(blocks_dev(b), out)
    ref = orc.dequant_q4k(b) if fmt == "q4k" else orc.dequant_q6k(b)
    assert host_bytes(out) == ref.tobytes()


def make_weights(orc, fmt, rows, cols, seed, adversarial=False):
    rng = Rng(seed)
    src = rng.adversarial(rows * cols) if adversarial else rng.vec(rows * cols)
    if fmt == "q8_0":
        return orc.q8_quantize(src)
    return orc.quantize_q4k_ref(src) if fmt == "q4k" else orc.quantize_q6k_ref(src)


def make_acts(orc, fmt, n, seed, batch=1):
    x = Rng(seed).vec(n * batch)
    return orc.q8_quantize(x) if fmt == "q8_0" else orc.quantize_q8k(x)


def gpu_matmul(K, fmt, w, xs, rows, cols, batch, w_offset=0):
    wb = np.frombuffer(w.tobytes(), np.uint8)
    if w_offset:
        wd = torch.empty(wb.size + 64, dtype=torch.uint8, device="cuda")
        wd[w_offset:w_offset + wb.size].copy_(dev(wb.copy()))
        wt = wd[w_offset:w_offset + wb.size]
    else:
        wt = dev(wb.copy())
    y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
    fn = {"q8_0": (K.matvec_q8, K.matmul_q8), "q4k": (K.matvec_q4k, K.matmul_q4k),
          "q6k": (K.matvec_q6k, K.matmul_q6k)}[fmt]
    if batch == 1:
        fn[0](y, wt, blocks_dev(xs), rows, cols)
    else:
        fn[1](y, wt, blocks_dev(xs), rows, cols, batch)
    K.sync_check()
    return y.cpu().numpy()


SHAPES = {
    "q8_0": [(48, 128), (48, 256), (7, 32), (33, 96), (2048, 2048), (512, 2048), (100, 8192), (64, 9728),
             (300, 2560)],
    "q4k": [(48, 512), (32, 512), (5, 256), (2048, 2048), (9728 // 64, 2560), (64, 9728), (37, 3072)],
    "q6k": [(32, 512), (3, 256), (2048, 2048), (70, 2560), (64, 9728), (41, 3072)],
}


@pytest.mark.parametrize("fmt", ["q8_0", "q4k", "q6k"])
def test_matvec_bit_exact_vs_scalar(K, orc, fmt):
    for i, (rows, cols) in enumerate(SHAPES[fmt]):
        w = make_weights(orc, fmt, rows, cols, 100 + i, adversarial=(i % 2 == 1))
        x = make_acts(orc, fmt, cols, 200 + i)
        ref = orc.matvec(fmt, w, x, rows, cols)
        got = gpu_matmul(K, fmt, w, x, rows, cols, 1)[0]
        assert got.tobytes() == ref.tobytes(), f"{fmt} {rows}x{cols}: max diff {np.max(np.abs(got - ref))}"


@pytest.mark.parametrize("fmt", ["q8_0", "q4k", "q6k"])
@pytest.mark.parametrize("batch", [2, 3, 5, 8, 9, 17, 64])
def test_matmul_bit_exact_and_equals_matvec(K, orc, fmt, batch):
    rows, cols = (96, 512) if fmt != "q8_0" else (96, 320)
    w = make_weights(orc, fmt, rows, cols, 7)
    xs = make_acts(orc, fmt, cols, 8, batch)
    ref = orc.matmul(fmt, w, xs, rows, cols, batch)
    got = gpu_matmul(K, fmt, w, xs, rows, cols, batch)
    assert got.tobytes() == ref.tobytes()
    bpr = cols // (32 if fmt == "q8_0" else 256)
    for b in range(batch):  # matmul == matvec, kernels.rs:277-292 / kquant.rs:297-329
        one = gpu_matmul(K, fmt, w, xs[b * bpr:(b + 1) * bpr].copy(), rows, cols, 1)[0]
        assert one.tobytes() == got[b].tobytes()


@pytest.mark.parametrize("batch", [1, 2, 3, 4])
@pytest.mark.parametrize("shape", [(100, 512), (33, 2048), (64, 8192), (1, 256), (2500, 512), (4099, 256),
                                   (4801, 2048)])
def test_matvec_q8_whole_octet_rows(K, orc, shape, batch):
    """Q8_0 rows of whole 16-byte aligned octets (cols % 256 == 0), 1-4 tokens:
    the streaming kernel with 32-octet stages (1, 2 or 4 octet columns of
    32, 16 or 8 rows: 4801 rows x 2048 fill every SM with 32-row groups, the
    small shapes take narrower groups), block terms chained in order by two
    chain warps. Partial last groups read zero-filled rows that are never
    stored."""
    rows, cols = shape
    w = make_weights(orc, "q8_0", rows, cols, 60 + rows + batch, adversarial=(batch % 2 == 0))
    xs = make_acts(orc, "q8_0", cols, 61 + batch, batch)
    ref = orc.matmul("q8_0", w, xs, rows, cols, batch)
    got = gpu_matmul(K, "q8_0", w, xs, rows, cols, batch)
    assert got.tobytes() == ref.tobytes(), f"{rows}x{cols} b{batch}: max diff {np.nanmax(np.abs(got - ref))}"


@pytest.mark.parametrize("shape", [(300, 2048), (130, 512), (2048, 2048), (64, 8192), (128, 256), (1, 768)])
@pytest.mark.parametrize("batch", [9, 16, 17, 33, 64, 100])
def test_matmul_q8_tensor_core_bit_exact(K, orc, shape, batch):
    """Q8_0 with cols % 256 == 0 and batch > 8 runs on tcgen05 (kind::i8, one
    MMA per block, scales applied in block order by the epilogue)."""
    rows, cols = shape
    w = make_weights(orc, "q8_0", rows, cols, 40 + rows, adversarial=(batch % 2 == 1))
    xs = make_acts(orc, "q8_0", cols, 41 + batch, batch)
    ref = orc.matmul("q8_0", w, xs, rows, cols, batch)
    got = gpu_matmul(K, "q8_0", w, xs, rows, cols, batch)
    if got.tobytes() != ref.tobytes():
        bad = np.argwhere(got.view(np.uint32) != ref.view(np.uint32))
        raise AssertionError(f"{rows}x{cols} b{batch}: {len(bad)} differ, first {bad[:4].tolist()}, "
                             f"max diff {np.nanmax(np.abs(got - ref))}")


@pytest.mark.parametrize("fmt", ["q4k", "q6k"])
@pytest.mark.parametrize("shape", [(5, 256), (37, 512), (133, 2560), (300, 3072), (128, 9728), (1000, 2048)])
@pytest.mark.parametrize("batch", [9, 33, 70])
def test_matmul_kquant_tensor_core_bit_exact(K, orc, fmt, shape, batch):
    """K-quant weights with more than 8 tokens run on tcgen05 (one kind::i8
    MMA per 32-value sub-block, Q6_K as masked 16-value halves). Rows come in
    8-row groups through a 2-D tensor map and the last rows % 8 by cp.async,
    so the shapes cover fewer than 8 rows, ragged tails, several 128-row tiles
    and super-block counts whose rows are not 16-byte multiples (Q6_K 10, 12,
    38 per row)."""
    rows, cols = shape
    w = make_weights(orc, fmt, rows, cols, 70 + rows + batch, adversarial=(batch % 2 == 1))
    xs = make_acts(orc, fmt, cols, 71 + batch, batch)
    ref = orc.matmul(fmt, w, xs, rows, cols, batch)
    got = gpu_matmul(K, fmt, w, xs, rows, cols, batch)
    if got.tobytes() != ref.tobytes():
        bad = np.argwhere(got.view(np.uint32) != ref.view(np.uint32))
        raise AssertionError(f"{fmt} {rows}x{cols} b{batch}: {len(bad)} differ, first {bad[:4].tolist()}")


@pytest.mark.parametrize("fmt", ["q8_0", "q4k", "q6k"])
@pytest.mark.parametrize("offset", [2, 4, 6, 8, 14])
def test_matvec_unaligned_weights(K, orc, fmt, offset):
    rows, cols = (37, 512)
    w = make_weights(orc, fmt, rows, cols, 31)
    x = make_acts(orc, fmt, cols, 32)
    ref = orc.matvec(fmt, w, x, rows, cols)
    got = gpu_matmul(K, fmt, w, x, rows, cols, 1, w_offset=offset)[0]
    assert got.tobytes() == ref.tobytes()


def test_saturated_blocks(K, orc):  # kquant.rs:210-245 blocks, bit-exact vs scalar
    from tests.test_oracle import saturated_blocks
    q4, q6 = saturated_blocks(orc)
    x = orc.quantize_q8k(Rng(81).adversarial(256))
    for fmt, blk in (("q4k", q4), ("q6k", q6)):
        w = np.concatenate([blk] * 16)
        ref = orc.matvec(fmt, w, x, 16, 256)
        got = gpu_matmul(K, fmt, w, x, 16, 256, 1)[0]
        assert got.tobytes() == ref.tobytes()
    # Q8_0 with -128 weight bytes (outside the quantizer's range, valid in GGUF files).
    w8 = np.zeros(64, O.Q8_0)
    w8["d"] = orc.f32_to_f16(np.array([0.75], np.float32))[0]
    w8["qs"] = -128
    x8 = orc.q8_quantize(Rng(5).adversarial(256))
    ref = orc.matvec("q8_0", w8, x8, 8, 256)
    got = gpu_matmul(K, "q8_0", w8, x8, 8, 256, 1)[0]
    assert got.tobytes() == ref.tobytes()


def test_matvec_empty_and_invalid(K):
    from nightrun_b200 import NrcError
    y = torch.empty(4, dtype=torch.float32, device="cuda")
    w = torch.zeros(34 * 4, dtype=torch.uint8, device="cuda")
    with pytest.raises(NrcError) as e:
        K.matvec_q8(y, w, w, 4, 33)
    assert e.value.name == "INVALID"
    K.matvec_q8(y, w, w, 0, 32)  # zero rows: no-op
    y.fill_(1.0)
    K.matvec_q8(y, w, w, 4, 0)  # zero cols: y = 0 like the empty dot
    assert torch.all(y == 0)


@pytest.mark.parametrize("n", [1, 31, 256, 2048, 8192, 9728])
def test_rmsnorm_softmax_swiglu_bit_exact(K, orc, n):
    rng = Rng(9 + n)
    x = rng.vec(n) * F(3)
    w = rng.vec(n) + F(1)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    K.rmsnorm(out, dev(x), dev(w), 1e-5)
    assert host_bytes(out) == orc.rmsnorm(x, w, 1e-5).tobytes()
    s = rng.vec(n) * F(8)
    st = dev(s)
    K.softmax(st)
    assert host_bytes(st) == orc.softmax(s).tobytes()
    g, u = rng.vec(n) * F(6), rng.vec(n)
    gt = dev(g)
    K.swiglu(gt, dev(u))
    assert host_bytes(gt) == orc.swiglu(g, u).tobytes()


def test_rmsnorm_softmax_rows(K, orc):
    rows, n = 5, 1000
    x = Rng(3).vec(rows * n) * F(4)
    w = Rng(4).vec(n)
    out = torch.empty(rows * n, dtype=torch.float32, device="cuda")
    K.rmsnorm(out, dev(x), dev(w), 1e-6, rows=rows)
    ref = np.concatenate([orc.rmsnorm(x[r * n:(r + 1) * n], w, 1e-6) for r in range(rows)])
    assert host_bytes(out) == ref.tobytes()
    st = dev(x)
    K.softmax(st, rows=rows)
    ref = np.concatenate([orc.softmax(x[r * n:(r + 1) * n]) for r in range(rows)])
    assert host_bytes(st) == ref.tobytes()


def test_expf_elementwise_matches_oracle(K, orc):
    r = np.random.default_rng(11)
    x = np.concatenate([
        r.integers(0, 2 ** 32, 1 << 20, dtype=np.uint64).astype(np.uint32).view(np.float32),
        r.uniform(-104.0, 89.0, 1 << 20).astype(np.float32),
        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 88.72283, 88.72284, -87.33655, -103.97208, -103.97209,
                  1e-8, -1e-8], np.float32),
    ])
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    K.expf(dev(x), y)
    got, ref = y.cpu().numpy(), orc.expf(x)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert got[~nan].tobytes() == ref[~nan].tobytes()


def test_expf_every_binary32_input(K):
    """Hashes of the device expf over all 2^32 inputs equal the oracle's, whose
    values were checked against long-double expl at generation time."""
    gold = np.fromfile(os.path.join(os.path.dirname(__file__), "golden", "expf_cr_hashes.bin"), np.uint64)
    out = torch.zeros(gold.size, dtype=torch.int64, device="cuda")
    K.expf_hash(out, 0, gold.size)
    K.sync_check()
    assert np.array_equal(out.cpu().numpy().view(np.uint64), gold)


def _sum_cases(n, seed):
    r = np.random.default_rng(seed)
    yield "normal", r.standard_normal(n).astype(F)
    yield "wide", (r.standard_normal(n) * np.exp(r.uniform(-20, 20, n))).astype(F)
    z = np.zeros(n, F)
    z[r.integers(0, n, 3)] = 1.5
    yield "mostly_zero", z
    yield "integers", r.integers(-3, 4, n).astype(F)  # many exact half-way additions
    yield "tiny", (r.standard_normal(n) * 1e-20).astype(F)  # subnormal squares
    big = r.standard_normal(n).astype(F)
    big[n // 2] = F(3e18)
    yield "one_huge", big


@pytest.mark.parametrize("n", [1, 63, 64, 65, 100, 1000, 2048, 4097, 8192, 8193, 20000])
def test_exact_parallel_sums_adversarial(K, orc, n):
    """rmsnorm's sum of squares and softmax's denominator (one pipelined
    serial chain on the device, 16-term blocks fetched ahead of their adds)
    must equal the reference's sequential chain bit for bit, on inputs chosen
    to stress binade crossings, half-way roundings, subnormals and a single
    dominating term."""
    w = (np.random.default_rng(n).standard_normal(n) + 1).astype(F)
    for name, x in _sum_cases(n, n + 7):
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        K.rmsnorm(out, dev(x), dev(w), 1e-5)
        assert host_bytes(out) == orc.rmsnorm(x, w, 1e-5).tobytes(), f"rmsnorm {name} n={n}"
        logits = (x / F(4)).astype(F)
        st = dev(logits)
        K.softmax(st)
        ref = orc.softmax(logits)
        got = st.cpu().numpy()
        assert got.tobytes() == ref.tobytes(), f"softmax {name} n={n}"


def test_argmax_first_max_and_edges(K):
    assert K.argmax(dev(np.array([0.1, 4.0, -2.0, 4.0], np.float32))) == 1  # kernels.rs:228-231
    assert K.argmax(dev(np.array([np.nan, -np.inf, 3.0, 3.0], np.float32))) == 2
    assert K.argmax(dev(np.array([np.nan, -np.inf], np.float32))) == 0
    assert K.argmax(dev(np.full(5, -np.inf, np.float32))) == 0
    big = np.random.default_rng(1).standard_normal(151936).astype(np.float32)
    big[100000] = big[5] = 99.0
    assert K.argmax(dev(big)) == 5


@pytest.mark.parametrize("style,hd", [(0, 64), (1, 128), (0, 128)])
def test_rope_bit_exact(K, orc, style, hd):
    freqs = K.rope_freqs(hd, 500000.0, (32.0, 1.0, 4.0, 8192.0))
    ref_f = orc.rope_freqs(hd, 500000.0, (32.0, 1.0, 4.0, 8192.0))
    assert np.array(freqs, np.float32).tobytes() == ref_f.tobytes()
    x = Rng(5).vec(hd * 6)
    for pos in (0, 1, 17, 4095):
        t = dev(x)
        K.rope_apply(t, hd, freqs, pos, style)
        assert host_bytes(t) == orc.rope_apply(x, hd, ref_f, pos, style).tobytes()


@pytest.mark.parametrize("kind", [0, 1])
def test_bounded_wait_expires_cleanly(K, orc, kind):
    """A wait that can never be satisfied (an mbarrier arrival withheld, or a
    flag nobody raises) gives up after its limit: the host gets NRC_ERR_DEVICE,
    the error word is cleared, and the next kernels run correctly."""
    import time
    from nightrun_b200 import NrcError, lib
    t0 = time.time()
    rc = lib().nrc_wait_selftest(kind, 20_000_000, None)  # 20 ms
    assert rc == -4, rc  # NRC_ERR_DEVICE
    assert time.time() - t0 < 5.0
    K.sync_check()  # cleared: no stale error
    w = make_weights(orc, "q8_0", 64, 512, 5)
    x = make_acts(orc, "q8_0", 512, 6)
    got = gpu_matmul(K, "q8_0", w, x, 64, 512, 1)[0]
    assert got.tobytes() == orc.matvec("q8_0", w, x, 64, 512).tobytes()
    with pytest.raises(NrcError):
        from nightrun_b200._lib import check
        check(lib().nrc_wait_selftest(2, 1000, None))
