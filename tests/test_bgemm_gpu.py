"""The batched-decode tensor-core GEMM (csrc/mlq_bgemm.cu) against the CPU
oracle, through the C ABI (mlq_linear routes 3..32 rows of x with
in_features % 32 == 0 to it).

Tolerance (the contract): relative L2 error of every output vector (row of
y) <= 1e-3.  Covered: every format; 3..32 rows (padded token counts 8, 16
and 32); partial row tiles; K extents that end inside a 256-value chunk;
matrices whose row tiles the work split cuts across CTAs (the fix-up pass),
at the BASELINE config-4 and config-5 shapes; the fused bias and SwiGLU
pair; NaN/Inf propagation; activations spanning six orders of magnitude in
one block, outlier channels, token rows of very different magnitudes and an
x that is not 16-byte aligned; and bit-identical repeats (the split and its fix-up are
deterministic)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2_rows

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def weights(oracle, pkg, fmt, out_f, in_f, seed):
    return oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=seed, std=0.02))


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
@pytest.mark.parametrize("shape", [(384, 1024), (300, 2048), (1000, 896), (4864, 896), (128, 32), (257, 4096)])
def test_bgemm_matches_oracle(oracle, pkg, fmt, shape):
    out_f, in_f = shape
    blocks = weights(oracle, pkg, fmt, out_f, in_f, seed=out_f + in_f)
    w = dev(blocks)
    for rows in (3, 4, 7, 8, 9, 16, 17, 32):
        assert pkg.mlq.takes_bgemm(rows, out_f, in_f)
        x = pkg.synth.normal((rows, in_f), seed=rows * 7 + in_f)
        y = pkg.mlq.linear(fmt, w, out_f, in_f, dev(x)).cpu().numpy()
        err = rel_l2_rows(y, oracle.linear(fmt, x, blocks, out_f)).max()
        assert err <= TOL, (fmt, shape, rows, err)
    assert pkg.mlq.device_error(0) == 0


@pytest.mark.parametrize("fmt,out_f,in_f,rows", [
    ("q8_0", 14336, 4096, 16),   # config 4: gate/up
    ("q8_0", 4096, 14336, 16),   # config 4: down
    ("q8_0", 1024, 4096, 16),    # config 4: k/v (fewer row tiles than SMs)
    ("q4_0", 28672, 8192, 8),    # config 5: gate/up at batch 8
    ("q4_0", 8192, 28672, 8),    # config 5: down at batch 8
])
def test_bgemm_baseline_shapes(oracle, pkg, fmt, out_f, in_f, rows):
    """Full-size BASELINE matrices: the work split cuts row tiles across CTAs
    and the fix-up pass sums them; checked on every output row."""
    blocks = weights(oracle, pkg, fmt, out_f, in_f, seed=11)
    x = pkg.synth.normal((rows, in_f), seed=12)
    w, xd = dev(blocks), dev(x)
    y = pkg.mlq.linear(fmt, w, out_f, in_f, xd)
    y2 = pkg.mlq.linear(fmt, w, out_f, in_f, xd)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)  # deterministic split and fix-up
    err = rel_l2_rows(y.cpu().numpy(), oracle.linear(fmt, x, blocks, out_f)).max()
    assert err <= TOL, err
    assert pkg.mlq.device_error(0) == 0


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
def test_bgemm_bias_and_swiglu(oracle, pkg, fmt):
    out_f, in_f, rows = 700, 2048, 12
    wg = weights(oracle, pkg, fmt, out_f, in_f, 21)
    wu = weights(oracle, pkg, fmt, out_f, in_f, 22)
    x = pkg.synth.normal((rows, in_f), seed=23)
    b = pkg.synth.normal((out_f,), seed=24, std=0.5)
    yb = pkg.mlq.linear_bias(fmt, dev(wg), out_f, in_f, dev(x), dev(b)).cpu().numpy()
    assert rel_l2_rows(yb, oracle.linear(fmt, x, wg, out_f) + b[None, :]).max() <= TOL
    h = pkg.mlq.linear_swiglu(fmt, dev(wg), dev(wu), out_f, in_f, dev(x)).cpu().numpy()
    ref = oracle.swiglu(oracle.linear(fmt, x, wg, out_f), oracle.linear(fmt, x, wu, out_f))
    assert rel_l2_rows(h, ref).max() <= TOL
    assert pkg.mlq.device_error(0) == 0


def test_bgemm_wide_dynamic_range(oracle, pkg):
    """One value per block 1e3, the rest ~1e-3 (the power-of-two token scale
    keeps every value to 2^-25 of the token's largest)."""
    fmt, out_f, in_f, rows = "q4_0", 384, 4096, 6
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 31)
    x = pkg.synth.normal((rows, in_f), seed=32, std=1e-3)
    x[:, ::32] = 1e3 * np.sign(x[:, ::32] + 1e-12)
    y = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, dev(x)).cpu().numpy()
    assert rel_l2_rows(y, oracle.linear(fmt, x, blocks, out_f)).max() <= TOL


@pytest.mark.parametrize("bad", [np.nan, np.inf])
def test_bgemm_non_finite_x_propagates(oracle, pkg, bad):
    fmt, out_f, in_f, rows = "q8_0", 256, 1024, 4
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 41)
    x = pkg.synth.normal((rows, in_f), seed=42)
    x[1, 100] = bad
    y = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, dev(x)).cpu().numpy()
    ref = oracle.linear(fmt, x, blocks, out_f)
    assert not np.isfinite(ref[1]).any() and not np.isfinite(y[1]).any()
    # the other rows of x are untouched by row 1's NaN / Inf
    assert rel_l2_rows(np.delete(y, 1, 0), np.delete(ref, 1, 0)).max() <= TOL


def test_bgemm_zero_x(oracle, pkg):
    fmt, out_f, in_f = "q4_1", 512, 2048
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 51)
    y = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, torch.zeros((5, in_f), device="cuda")).cpu().numpy()
    np.testing.assert_array_equal(y, np.zeros((5, out_f), np.float32))


def test_bgemm_outliers_and_token_magnitudes(oracle, pkg):
    """Decoder activations carry a few outlier channels ~1000x the rest; the
    tokens of a batch may differ by many orders of magnitude (each token has
    its own power-of-two scale, applied after the sum)."""
    fmt, out_f, in_f, rows = "q8_0", 1000, 4096, 9
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 61)
    x = pkg.synth.normal((rows, in_f), seed=62)
    x[:, [7, 1000, 2049, 4000]] *= 2000.0
    x[2] *= 1e-30
    x[3] *= 1e30
    x[4] *= 2.0 ** -100
    x[5] = 0.0
    y = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, dev(x)).cpu().numpy()
    ref = oracle.linear(fmt, x, blocks, out_f)
    assert np.isfinite(y).all()
    np.testing.assert_array_equal(y[5], np.zeros(out_f, np.float32))
    keep = [r for r in range(rows) if r != 5]
    assert rel_l2_rows(y[keep], ref[keep]).max() <= TOL
    assert pkg.mlq.device_error(0) == 0


@pytest.mark.parametrize("fmt", ["q4_0", "q4_1"])
def test_bgemm_unaligned_x(oracle, pkg, fmt):
    """x starting 4 bytes past a 16-byte boundary (a view into a larger
    buffer) is read element by element."""
    out_f, in_f, rows = 640, 1024, 5
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 71)
    x = pkg.synth.normal((rows, in_f), seed=72)
    buf = torch.empty(rows * in_f + 1, device="cuda")
    xv = buf[1:].view(rows, in_f)
    xv.copy_(dev(x))
    assert xv.data_ptr() % 16 == 4
    y = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, xv).cpu().numpy()
    assert rel_l2_rows(y, oracle.linear(fmt, x, blocks, out_f)).max() <= TOL
    assert pkg.mlq.device_error(0) == 0
