"""nrc_matmul_q8_0_noalloc (static device scratch, no allocation) against the
existing nrc_matmul_q8_0 on the same inputs, over two consecutive calls that
reuse the scratch: the tensor-core path (batch > 8, cols % 256 == 0) and the
GEMV path (batch <= 8 or ragged cols). This file is named to be collected
last; it passes alone and after the other GPU tests."""
import numpy as np
import pytest
import torch

from tests.refdata import Rng

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from nightrun_b200 import kernels
    return kernels


def dev_bytes(blocks):
    return torch.from_numpy(np.frombuffer(blocks.tobytes(), np.uint8).copy()).cuda()


def run(fn, w, xs, rows, cols, batch):
    y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
    fn(y, dev_bytes(w), dev_bytes(xs), rows, cols, batch)
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("rows,cols,batch", [(300, 2048, 64), (130, 512, 17), (2048, 8192, 33), (96, 320, 5),
                                             (64, 16384, 100), (7, 96, 9)])
def test_noalloc_matches_matmul_q8_over_two_calls(K, orc, rows, cols, batch):
    w = orc.q8_quantize(Rng(rows + cols).vec(rows * cols))
    for call in range(2):
        xs = orc.q8_quantize(Rng(1000 * call + batch).vec(cols * batch))
        ref = run(K.matmul_q8, w, xs, rows, cols, batch)
        got = run(K.matmul_q8_noalloc, w, xs, rows, cols, batch)
        assert got.tobytes() == ref.tobytes(), f"call {call}: {rows}x{cols} b{batch}"
        if rows * cols * batch <= 2048 * 8192 * 33:
            # and directly against the reference's scalar matmul (kernels.rs:91-143)
            want = orc.matmul("q8_0", w, xs, rows, cols, batch).reshape(batch, rows)
            assert got.tobytes() == want.tobytes(), f"call {call}: {rows}x{cols} b{batch} vs oracle"


def test_noalloc_rejects_cols_beyond_scratch(K):
    from nightrun_b200 import NrcError
    cols = K_MAX = 16384 + 32
    y = torch.empty(4, dtype=torch.float32, device="cuda")
    w = torch.zeros(4 * K_MAX // 32 * 34, dtype=torch.uint8, device="cuda")
    x = torch.zeros(K_MAX // 32 * 34, dtype=torch.uint8, device="cuda")
    with pytest.raises(NrcError) as e:
        K.matmul_q8_noalloc(y, w, x, 4, cols, 1)
    assert e.value.name == "INVALID"
    assert "scratch" in str(e.value)
