"""CPU tests of the oracle (oracle/oracle.c): pinned against the reference's
own outputs (tests/golden/reference_quant.npz, made by make_golden.py from
the reference's compiled src/quant.cc) and the reference's known-answer
tests (tests/test_quant.cc)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_quant.npz"
SHAPES = [(4, 32), (7, 100), (3, 96), (8, 1024), (5, 1), (2, 33), (6, 64)]


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# --- golden vectors: bit-exact -------------------------------------------------------------
@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("shape", SHAPES)
def test_quantize_dequantize_linear_match_reference(oracle, golden, fmt, shape):
    rows, cols = shape
    key = f"{fmt}_{rows}x{cols}"
    blocks = oracle.quantize(fmt, golden[f"{key}_w"])
    assert np.array_equal(blocks, golden[f"{key}_blocks"]), "quantized bytes differ"
    deq = oracle.dequantize(fmt, blocks, rows, cols)
    assert np.array_equal(bits(deq), bits(golden[f"{key}_deq"]))
    for xr in (0, 3):
        y = oracle.linear(fmt, golden[f"{key}_x{xr}"], blocks, rows)
        assert np.array_equal(bits(y), bits(golden[f"{key}_y{xr}"])), (key, xr)


@pytest.mark.parametrize("shape", SHAPES)
def test_q4_1_dequantize_linear_match_reference(oracle, golden, shape):
    rows, cols = shape
    key = f"q4_1_{rows}x{cols}"
    blocks = golden[f"{key}_blocks"]
    assert np.array_equal(bits(oracle.dequantize("q4_1", blocks, rows, cols)), bits(golden[f"{key}_deq"]))
    for xr in (0, 3):
        y = oracle.linear("q4_1", golden[f"{key}_x{xr}"], blocks, rows)
        assert np.array_equal(bits(y), bits(golden[f"{key}_y{xr}"]))


def test_reference_gpu_test_inputs(oracle, golden):
    """The fillLinear cases of the reference's tests/test_cuda.cc:679-743."""
    for fmt in ("q8_0", "q4_0"):
        b = oracle.quantize(fmt, golden["tc_w"])
        assert np.array_equal(b, golden[f"tc_{fmt}_blocks"])
        assert np.array_equal(bits(oracle.linear(fmt, golden["tc_x"], b, 4)), bits(golden[f"tc_{fmt}_y"]))
        assert np.array_equal(bits(oracle.linear(fmt, golden["tc_x2"], b, 4)), bits(golden[f"tc_{fmt}_y2"]))
    y = oracle.linear("q4_1", golden["tc_x"], golden["tc_q4_1_blocks"], 4)
    assert np.array_equal(bits(y), bits(golden["tc_q4_1_y"]))


def test_swiglu_matches_reference(oracle, golden):
    """orc_swiglu against the reference's swiGlu (src/ops.cc:111-145), gate
    values -100..100 (exp overflow / underflow) and random ones: bit-exact."""
    h = oracle.swiglu(golden["swiglu_gate"], golden["swiglu_up"])
    assert np.array_equal(bits(h), bits(golden["swiglu_h"]))


def test_gate_up_pair_matches_reference(oracle, golden):
    """The SwiGLU of two q4_0 linears sharing x (ffnForwardDevice's gate, up
    and forwardSwiGluDevice, src/forward.cc:573-581): oracle linear + swiglu
    reproduces the reference's outputs bit for bit."""
    x = golden["ffn_x"]
    g = oracle.linear("q4_0", x, golden["ffn_gate_blocks"], 48)
    u = oracle.linear("q4_0", x, golden["ffn_up_blocks"], 48)
    assert np.array_equal(bits(oracle.swiglu(g, u)), bits(golden["ffn_h"]))


def test_add_bias_matches_host_add(oracle, golden):
    """orc_add_bias = the reference host variants' y[r][c] += bias[c]
    (src/cuda_quant.cu:326-329) on the reference GPU tests' bias."""
    y = golden["tc_q8_0_y2"]
    out = oracle.add_bias(y, golden["tc_bias"])
    assert np.array_equal(bits(out), bits((y + golden["tc_bias"][None, :]).astype(np.float32)))
    assert np.array_equal(bits(y), bits(golden["tc_q8_0_y2"]))  # input untouched


# --- the reference's known-answer tests (tests/test_quant.cc) ------------------------------
def test_block_layout(pkg):
    # test_quant.cc:11-15, 184-194
    from oracle.oracle import BLOCK_BYTES
    assert BLOCK_BYTES == {"q8_0": 34, "q4_0": 18, "q4_1": 20}
    assert pkg.mlq.BLOCK_BYTES == BLOCK_BYTES


def test_q8_0_roundtrip_identity(oracle):
    # test_quant.cc:20-44
    src = (np.arange(32, dtype=np.float32) * np.float32(0.1)).reshape(1, 32)
    blocks = oracle.quantize("q8_0", src)
    assert blocks.size == 34
    assert np.abs(oracle.dequantize("q8_0", blocks, 1, 32) - src).max() < 6e-2


def test_q8_0_all_zeros(oracle):
    # test_quant.cc:46-56
    blocks = oracle.quantize("q8_0", np.zeros((1, 64), np.float32))
    assert blocks.size == 68 and not blocks.any()
    assert np.abs(oracle.dequantize("q8_0", blocks, 1, 64)).max() <= 1e-6


def test_q8_0_multi_block(oracle):
    # test_quant.cc:58-79
    src = (np.arange(100, dtype=np.float32) * np.float32(0.05)).reshape(1, 100)
    blocks = oracle.quantize("q8_0", src)
    assert blocks.size == 4 * 34
    assert np.abs(oracle.dequantize("q8_0", blocks, 1, 100) - src).max() < 6e-2


def test_q4_0_roundtrip_and_zeros(oracle):
    # test_quant.cc:196-229
    src = (np.arange(32, dtype=np.float32) * np.float32(0.1)).reshape(1, 32)
    b = oracle.quantize("q4_0", src)
    assert b.size == 18
    assert np.abs(oracle.dequantize("q4_0", b, 1, 32) - src).max() < 3e-1
    z = oracle.quantize("q4_0", np.zeros((1, 64), np.float32))
    assert np.abs(oracle.dequantize("q4_0", z, 1, 64)).max() <= 1e-6


def q41_block(d: int, m: int, qs) -> np.ndarray:
    b = np.zeros(20, np.uint8)
    b[0], b[1], b[2], b[3] = d & 0xFF, d >> 8, m & 0xFF, m >> 8
    b[4:20] = np.asarray(qs, np.uint8)
    return b


def test_q4_1_dequantize_known_values(oracle):
    # test_quant.cc:231-248: d = 0.5, m = -1, nibbles i | (15-i) << 4
    b = q41_block(0x3800, 0xBC00, [i | ((15 - i) << 4) for i in range(16)])
    w = oracle.dequantize("q4_1", b, 1, 32)[0]
    assert np.allclose(w[:16], -1.0 + 0.5 * np.arange(16), atol=1e-6)
    assert np.allclose(w[16:], -1.0 + 0.5 * (15 - np.arange(16)), atol=1e-6)


def test_q4_1_linear_known_values(oracle):
    # test_quant.cc:250-263: all nibbles 1, d = 1, m = 0, x = 2  ->  64
    b = q41_block(0x3C00, 0x0000, [0x11] * 16)
    y = oracle.linear("q4_1", np.full(32, 2.0, np.float32), b, 1)
    assert y.shape == (1,) and abs(float(y[0]) - 64.0) <= 1e-6


def test_q4_0_linear_matches_f32(oracle):
    # test_quant.cc:265-286
    w = (np.arange(128, dtype=np.float32) * np.float32(0.05) - np.float32(1.0)).reshape(4, 32)
    x = np.arange(32, dtype=np.float32) * np.float32(0.1) - np.float32(0.4)
    yq = oracle.linear("q4_0", x, oracle.quantize("q4_0", w), 4)
    assert np.abs(yq - w @ x).max() <= 2.0


# --- fp16 encoder rounding rule (src/quant.cc:32-70) ---------------------------------------
def test_fp16_encoder_rounding_rule(oracle):
    enc = oracle.fp16_from_f32
    assert enc(0.5) == 0x3800 and enc(-1.0) == 0xBC00 and enc(1.0) == 0x3C00
    # 1 + 2^-11 is exactly halfway between fp16 1.0 and 1.0 + 2^-10: the
    # reference rounds half UP (0x3C01); round-to-nearest-even would give 0x3C00.
    assert enc(1.0 + 2.0 ** -11) == 0x3C01
    assert enc(65504.0) == 0x7BFF and enc(1e6) == 0x7C00 and enc(-1e6) == 0xFC00
    assert enc(float("nan")) == 0x7C00  # NaN encodes as +Inf
    assert enc(2.0 ** -24) == 0x0001 and enc(2.0 ** -26) == 0x0000
    for h in (0x0001, 0x03FF, 0x0400, 0x3555, 0x7BFF, 0x8001, 0xFBFF):
        assert enc(oracle.f32_from_fp16(h)) == h  # exact round trip of every fp16 value tried


# --- oracle vs the reference build, random shapes (only where oracle/_ref exists) ----------
@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_oracle_matches_reference_build_random(oracle, reference, pkg, fmt):
    rng = np.random.default_rng(7)
    for trial in range(6):
        rows = int(rng.integers(1, 40))
        cols = int(rng.integers(1, 700))
        w = pkg.synth.normal((rows, cols), seed=50 + trial, std=0.02)
        bo, br = oracle.quantize(fmt, w), reference.quantize(fmt, w)
        assert np.array_equal(bo, br)
        x = pkg.synth.normal((3, cols), seed=60 + trial)
        assert np.array_equal(bits(oracle.linear(fmt, x, bo, rows)), bits(reference.linear(fmt, x, br, rows)))


@pytest.mark.parametrize("src", ["q8_0", "q4_0"])
@pytest.mark.parametrize("dst", ["q8_0", "q4_0"])
def test_requantize_rule_matches_reference(oracle, reference, pkg, src, dst):
    """The oracle's dequantize-then-quantize (the GPU transcode's checker)
    equals the reference's own dequantizeFrom* + quantizeTo* (its
    quantizeQtToQ80/Q40 rule, src/model.cc:94-149) byte for byte."""
    rows, cols = 9, 100
    w = pkg.synth.normal((rows, cols), seed=5, std=0.02)
    b = reference.quantize(src, w)
    mine = oracle.quantize(dst, oracle.dequantize(src, b, rows, cols))
    ref = reference.quantize(dst, reference.dequantize(src, b, rows, cols))
    np.testing.assert_array_equal(mine, ref)
