"""GPU parity tests: libmlq.so (through the C ABI) against the CPU oracle.

Tolerance (the contract): relative L2 error of every output vector (row of
y) <= 1e-3, because the GPU sums in a different fp32 order than the
reference's sequential loop.  Dequantized weights and quantized blocks must
be bit-identical.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2_rows

pytestmark = pytest.mark.gpu
TOL = 1e-3

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_weights(oracle, pkg, fmt, out_f, in_f, seed):
    w = pkg.synth.normal((out_f, in_f), seed=seed, std=0.02)
    return oracle.quantize(fmt, w)


def gpu_linear(pkg, fmt, blocks, out_f, in_f, x):
    y = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, dev(x))
    torch.cuda.synchronize()
    return y.cpu().numpy()


SMALL = [(4, 32), (1, 32), (3, 100), (37, 96), (5, 1), (64, 4096), (200, 3584), (33, 18944),
         (300, 896), (17, 2080)]


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
@pytest.mark.parametrize("shape", SMALL)
def test_linear_matches_oracle(oracle, pkg, fmt, shape):
    out_f, in_f = shape
    blocks = make_weights(oracle, pkg, fmt, out_f, in_f, seed=out_f * 7 + in_f)
    for rows in (1, 2, 3, 5, 8, 16):
        x = pkg.synth.normal((rows, in_f), seed=rows + in_f)
        y = gpu_linear(pkg, fmt, blocks, out_f, in_f, x)
        ref = oracle.linear(fmt, x, blocks, out_f)
        err = rel_l2_rows(y, ref).max()
        assert err <= TOL, (fmt, shape, rows, err)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
def test_one_dimensional_x(oracle, pkg, fmt):
    blocks = make_weights(oracle, pkg, fmt, 96, 640, seed=3)
    x = pkg.synth.normal((640,), seed=4)
    y = gpu_linear(pkg, fmt, blocks, 96, 640, x)
    assert y.shape == (96,)
    assert rel_l2_rows(y, oracle.linear(fmt, x, blocks, 96)).max() <= TOL


# The BASELINE.json matrices at full size (weights N(0,0.02), x N(0,1)).
CONFIG_MATRICES = [
    ("q8_0", 4864, 896, 1),      # config 1
    ("q4_0", 4608, 3584, 1),     # config 2: QKV
    ("q4_0", 3584, 3584, 1),     # O
    ("q4_0", 18944, 3584, 1),    # gate / up
    ("q4_0", 3584, 18944, 1),    # down
    ("q4_0", 152064, 3584, 1),   # lm_head
    ("q8_0", 14336, 4096, 16),   # config 4: FFN, batch 16
    ("q8_0", 4096, 14336, 16),
    ("q4_0", 28672, 8192, 8),    # config 5: 70B FFN, batch 8
    ("q4_0", 8192, 28672, 1),
]


@pytest.mark.parametrize("fmt,out_f,in_f,rows", CONFIG_MATRICES)
def test_config_matrices_full_size(oracle, pkg, fmt, out_f, in_f, rows):
    blocks = make_weights(oracle, pkg, fmt, out_f, in_f, seed=11)
    x = pkg.synth.normal((rows, in_f), seed=12)
    w_d, x_d = dev(blocks), dev(x)
    y = pkg.mlq.linear(fmt, w_d, out_f, in_f, x_d)
    ref = oracle.linear(fmt, x, blocks, out_f)
    err = rel_l2_rows(y.cpu().numpy(), ref).max()
    assert err <= TOL, err
    # size-independent property: y(2x) == 2 y(x) exactly (power-of-two scaling)
    y2 = pkg.mlq.linear(fmt, w_d, out_f, in_f, x_d * 2)
    assert torch.equal(y2, y * 2)


def test_prefill_rows_q4_1(oracle, pkg):
    """Config 3 shape (x 512 x 4096 against 14336 x 4096); rows of y depend
    only on their row of x, so the oracle checks a sample of rows."""
    fmt, out_f, in_f, rows = "q4_1", 14336, 4096, 512
    blocks = make_weights(oracle, pkg, fmt, out_f, in_f, seed=21)
    x = pkg.synth.normal((rows, in_f), seed=22)
    y = gpu_linear(pkg, fmt, blocks, out_f, in_f, x)
    pick = [0, 1, 63, 64, 255, 511]
    ref = oracle.linear(fmt, x[pick], blocks, out_f)
    assert rel_l2_rows(y[pick], ref).max() <= TOL


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
def test_unaligned_weight_pointer(oracle, pkg, fmt):
    """Weights at a 2-byte offset (the blocks' own alignment) take the
    any-alignment path; a 16-byte offset keeps the streaming path."""
    out_f, in_f = 70, 1024
    blocks = make_weights(oracle, pkg, fmt, out_f, in_f, seed=5)
    x = pkg.synth.normal((3, in_f), seed=6)
    ref = oracle.linear(fmt, x, blocks, out_f)
    x_d = dev(x)  # keep every device buffer referenced until the kernel has run
    for off in (2, 16):
        buf = torch.zeros(blocks.size + 64, dtype=torch.uint8, device="cuda")
        buf[off:off + blocks.size] = dev(blocks)
        y = torch.empty((3, out_f), dtype=torch.float32, device="cuda")
        pkg.mlq.linear_raw(fmt, buf.data_ptr() + off, blocks.size // pkg.mlq.BLOCK_BYTES[fmt], out_f,
                           in_f, x_d.data_ptr(), 3, y.data_ptr(),
                           torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert rel_l2_rows(y.cpu().numpy(), ref).max() <= TOL, off


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
def test_output_guard_and_overwrite(oracle, pkg, fmt):
    """y is overwritten, never accumulated into, and nothing outside it is written."""
    out_f, in_f, rows = 130, 2048, 3
    blocks = make_weights(oracle, pkg, fmt, out_f, in_f, seed=8)
    x = pkg.synth.normal((rows, in_f), seed=9)
    guard = 256
    buf = torch.full((rows * out_f + 2 * guard,), 12345.0, dtype=torch.float32, device="cuda")
    w_d, x_d = dev(blocks), dev(x)  # held until the kernel has run (caching allocator reuse)
    pkg.mlq.linear_raw(fmt, w_d.data_ptr(), blocks.size // pkg.mlq.BLOCK_BYTES[fmt], out_f,
                       in_f, x_d.data_ptr(), rows, buf.data_ptr() + guard * 4,
                       torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    h = buf.cpu().numpy()
    assert (h[:guard] == 12345.0).all() and (h[-guard:] == 12345.0).all()
    y = h[guard:-guard].reshape(rows, out_f)
    assert rel_l2_rows(y, oracle.linear(fmt, x, blocks, out_f)).max() <= TOL


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
@pytest.mark.parametrize("shape", [(4, 32), (7, 100), (130, 4096), (9, 96)])
def test_dequantize_bit_exact(oracle, pkg, fmt, shape):
    out_f, in_f = shape
    blocks = make_weights(oracle, pkg, fmt, out_f, in_f, seed=13)
    got = pkg.mlq.dequantize(fmt, dev(blocks), out_f, in_f).cpu().numpy()
    want = oracle.dequantize(fmt, blocks, out_f, in_f)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
@pytest.mark.parametrize("shape", [(4, 32), (7, 100), (300, 4096), (3, 1), (5, 33)])
def test_quantize_bit_exact(oracle, pkg, fmt, shape):
    rows, cols = shape
    w = pkg.synth.normal((rows, cols), seed=rows + cols, std=0.02)
    w[0, 0] = 0.0
    if rows > 1:
        w[1, :] = 0.0  # an all-zero row
    got = pkg.mlq.quantize(fmt, dev(w)).cpu().numpy()
    assert np.array_equal(got, oracle.quantize(fmt, w))


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
def test_host_entry_points_with_bias(oracle, pkg, fmt):
    out_f, in_f, rows = 50, 512, 2
    blocks = make_weights(oracle, pkg, fmt, out_f, in_f, seed=14)
    x = pkg.synth.normal((rows, in_f), seed=15)
    bias = pkg.synth.normal((out_f,), seed=16)
    ref = oracle.linear(fmt, x, blocks, out_f) + bias
    y1 = pkg.mlq.linear_host(fmt, dev(blocks), out_f, in_f, x, bias)
    y2 = pkg.mlq.linear_host_weight(fmt, blocks, out_f, in_f, x, bias)
    assert rel_l2_rows(y1, ref).max() <= TOL
    assert np.array_equal(y1, y2)


def test_non_default_stream_and_determinism(oracle, pkg):
    fmt, out_f, in_f = "q4_0", 1000, 3584
    blocks = make_weights(oracle, pkg, fmt, out_f, in_f, seed=17)
    x = pkg.synth.normal((1, in_f), seed=18)
    s = torch.cuda.Stream()
    w_d, x_d = dev(blocks), dev(x)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        ya = pkg.mlq.linear(fmt, w_d, out_f, in_f, x_d, stream=s)
        yb = pkg.mlq.linear(fmt, w_d, out_f, in_f, x_d, stream=s)
    s.synchronize()
    assert torch.equal(ya, yb)  # no atomics: bit-identical repeats
    assert rel_l2_rows(ya.cpu().numpy(), oracle.linear(fmt, x, blocks, out_f)).max() <= TOL


def test_no_device_error_recorded(pkg):
    assert pkg.mlq.device_error(0) == 0


@pytest.mark.parametrize("fmt,out_f,in_f,rows", [("q4_0", 4608, 3584, 1), ("q8_0", 1000, 1024, 3),
                                                  ("q4_1", 512, 4096, 16)])
def test_host_entry_pinned_buffers(oracle, pkg, fmt, out_f, in_f, rows):
    """mlq_linear_host with pinned x/y (the bench's e2e path, asynchronous DMA)
    gives the same values as with pageable buffers, with and without the
    host bias."""
    blocks = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=out_f + rows, std=0.02))
    w = torch.from_numpy(blocks).cuda()
    x = pkg.synth.normal((rows, in_f), seed=rows + 40)
    bias = pkg.synth.normal((out_f,), seed=41, std=0.5)
    y_page = pkg.mlq.linear_host(fmt, w, out_f, in_f, x)
    yt = torch.full((rows, out_f), float("nan"), dtype=torch.float32).pin_memory()
    y_pin = pkg.mlq.linear_host(fmt, w, out_f, in_f, x, y=yt.numpy())
    assert np.array_equal(y_pin, y_page)
    assert rel_l2_rows(y_pin, oracle.linear(fmt, x, blocks, out_f)).max() <= TOL
    yb_page = pkg.mlq.linear_host(fmt, w, out_f, in_f, x, bias=bias)
    ybt = torch.zeros((rows, out_f), dtype=torch.float32).pin_memory()
    yb_pin = pkg.mlq.linear_host(fmt, w, out_f, in_f, x, bias=bias, y=ybt.numpy())
    assert np.array_equal(yb_pin, yb_page)
    assert pkg.mlq.device_error(0) == 0
