"""The tensor-core GEMM path against the CPU oracle (calls with >= 9 rows of
x, or >= 5 rows on matrices of >= 2^25 weights: MLQ_GEMM_ROWS_RULE), with and
without split-K (ranges of whole 256-value weight chunks when the output
tiles cannot fill the SMs).

Same contract as the GEMV: relative L2 error of every output row <= 1e-3.
The bf16x3 split keeps the GEMM within ~1e-5 of fp32, so the tests also
check a tighter 1e-4 to catch a lost split term.  Shapes cover partial
tiles in every dimension (out % 128, tokens % 128, in % 64 / % 256)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2_rows

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


CASES = [
    ("q4_1", 300, 1024, 64),
    ("q4_0", 256, 2048, 128),
    ("q8_0", 200, 4096, 100),
    ("q4_0", 1000, 3584, 200),
    ("q4_1", 129, 96, 65),       # in: one full and one partial 64-wide K-step
    ("q8_0", 384, 1280, 256),    # in: 5 K-chunks of 256
    ("q4_1", 640, 4160, 96),     # in % 256 = 64
    ("q8_0", 512, 4096, 16),     # batched decode
    ("q8_0", 512, 4096, 9),      # smallest GEMM row count on a narrow matrix
    ("q4_0", 12288, 4096, 5),    # large matrix: the GEMM from 5 rows
    ("q4_1", 12300, 3072, 7),    # large, partial last row tile
    ("q8_0", 1024, 8192, 16),    # 8 row tiles: split-K into 8 ranges of 4 weight chunks
    ("q4_0", 640, 4864, 12),     # 5 row tiles, 19 weight chunks: 7 ranges, the last of 1 chunk
    ("q4_0", 300, 2048, 20),
    ("q4_1", 256, 1024, 33),
    ("q8_0", 384, 1024, 24),     # 32-wide tile, stage count trimmed to fit shared memory
    ("q4_0", 200, 3584, 48),     # 64-wide tile
]


@pytest.mark.parametrize("fmt,out_f,in_f,rows", CASES)
def test_gemm_matches_oracle(oracle, pkg, fmt, out_f, in_f, rows):
    blocks = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=out_f + in_f, std=0.02))
    x = pkg.synth.normal((rows, in_f), seed=rows)
    w_d, x_d = dev(blocks), dev(x)
    y = pkg.mlq.linear(fmt, w_d, out_f, in_f, x_d)
    torch.cuda.synchronize()
    err = rel_l2_rows(y.cpu().numpy(), oracle.linear(fmt, x, blocks, out_f)).max()
    assert err <= 1e-4, err  # contract: 1e-3; the split GEMM reaches ~1e-5
    assert pkg.mlq.device_error(0) == 0


@pytest.mark.parametrize("fmt,out_f,in_f", [("q4_1", 14336, 4096), ("q4_1", 4096, 14336)])
def test_config3_prefill_rows(oracle, pkg, fmt, out_f, in_f):
    """BASELINE config 3 (x 512 x 4096 / 512 x 14336, q4_1): the oracle checks a
    sample of rows (each row of y depends only on its row of x)."""
    rows = 512
    blocks = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=5, std=0.02))
    x = pkg.synth.normal((rows, in_f), seed=6)
    y = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, dev(x)).cpu().numpy()
    pick = [0, 1, 127, 128, 300, 511]
    err = rel_l2_rows(y[pick], oracle.linear(fmt, x[pick], blocks, out_f)).max()
    assert err <= 1e-4, err
    # size-independent property over all 512 rows: y(2x) == 2 y(x) exactly
    y2 = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, dev(x * 2)).cpu().numpy()
    assert np.array_equal(y2, 2 * y)


def test_gemm_and_gemv_agree(oracle, pkg):
    """Rows 0..63 through the GEMM and the same rows 8 at a time through the
    GEMV: both within the contract of each other."""
    fmt, out_f, in_f = "q4_0", 512, 2048
    blocks = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=9, std=0.02))
    x = pkg.synth.normal((64, in_f), seed=10)
    w_d = dev(blocks)
    yg = pkg.mlq.linear(fmt, w_d, out_f, in_f, dev(x)).cpu().numpy()
    yv = np.concatenate([pkg.mlq.linear(fmt, w_d, out_f, in_f, dev(x[i:i + 8])).cpu().numpy()
                         for i in range(0, 64, 8)])
    assert rel_l2_rows(yg, yv).max() <= 1e-4
