"""CPU-side checks of the CUDA library (no GPU needed): the C ABI loads and
exports every entry point include/nrcuda.h declares, the host-side .nrm parser
rejects every malformed file the reference's tests build, and host-computed
RoPE frequencies equal the reference restatement bit for bit."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from tests.refdata import malformed_cases, tiny_nrm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def L():
    from nightrun_b200 import _lib
    so = _lib.LIB_PATH
    if not os.path.exists(so):
        from nightrun_b200 import build
        build.build()
    return _lib.lib()


def header_functions():
    text = open(os.path.join(ROOT, "include", "nrcuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nrc_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_exported_and_bound(L):
    from nightrun_b200 import _lib
    names = header_functions()
    assert len(names) > 30
    bound = {n for n, _, _ in _lib.SIGNATURES}
    for n in names:
        assert hasattr(L, n), f"{n} not exported by libnrcuda.so"
        assert n in bound, f"{n} has no ctypes signature"
    assert L.nrc_version() >= 100


def _load(L, blob):
    buf = np.frombuffer(bytes(blob), np.uint8).copy() if len(blob) else np.zeros(1, np.uint8)
    h = C.c_void_p()
    rc = L.nrc_model_load(buf.ctypes.data_as(C.c_void_p), len(blob), 0, 1, C.byref(h))
    return rc


@pytest.mark.parametrize("name,blob,meta_crc", malformed_cases(), ids=[c[0] for c in malformed_cases()])
def test_parser_rejects_malformed(L, name, blob, meta_crc):  # format_malformed.rs:110-206
    rc = _load(L, blob)
    assert rc in (-10, -11, -12, -13, -14), f"{name}: rc {rc}"
    if meta_crc:
        assert rc == -13


def test_parser_accepts_valid_file(L):
    # A valid file parses; without a GPU the upload step then fails cleanly.
    rc = _load(L, tiny_nrm())
    assert rc in (0, -2, -3)


def test_rope_freqs_host_bit_exact(L, orc):
    for hd, theta, sc in [(64, 500000.0, (32.0, 1.0, 4.0, 8192.0)), (128, 5e6, None), (64, 1e4, None),
                          (128, 500000.0, (32.0, 1.0, 4.0, 8192.0))]:
        out = (C.c_float * (hd // 2))()
        f, lo, hi, orig = sc if sc else (0.0, 0.0, 0.0, 0.0)
        assert L.nrc_rope_freqs(out, hd, theta, f, lo, hi, orig) == 0
        assert np.array(out, np.float32).tobytes() == orc.rope_freqs(hd, theta, sc).tobytes()


def test_invalid_arguments_rejected_without_gpu(L):
    assert L.nrc_matvec_q8_0(None, None, None, 4, 33, None) == -1
    assert L.nrc_quantize_q8k(None, None, 100, None) == -1
    assert L.nrc_ctx_forward(None, 0, None, None) == -1
    assert b"null" in L.nrc_last_error()


def test_noalloc_limits_checked_before_any_device_call(L):
    # Argument validation of the no-allocation matmul runs on the host only.
    fake = C.c_void_p(0x1000)
    assert L.nrc_matmul_q8_0_noalloc(fake, fake, fake, 4, 16384 + 32, 2, None) == -1
    assert b"scratch" in L.nrc_last_error()
    assert L.nrc_matmul_q8_0_noalloc(fake, fake, fake, 4, 33, 2, None) == -1
