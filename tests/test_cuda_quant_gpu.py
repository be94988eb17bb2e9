"""The reference's own quantized-linear GPU tests (tests/test_cuda.cc:679-809),
re-expressed against the reference-named entry points of
mini-llama_b200/cuda_quant.py, with the same inputs and tolerances.  The CPU
side of each comparison is the reference's linearQ80/Q40/Q41 output,
recorded in tests/golden/reference_quant.npz."""
from __future__ import annotations

import importlib
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_quant.npz"


@pytest.fixture(scope="module")
def cq(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return importlib.import_module("mini_llama_b200.cuda_quant")


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def expect_near(actual, expected, tol):
    """The reference's max-abs check (tests/test_cuda.cc:80-103), scaled by the
    output magnitude when it exceeds 1: the reference's GPU kernel passes an
    absolute 1e-4 only because it sums in the CPU's order; this library sums
    in a different fp32 order (the contract bounds that by relative L2 1e-3),
    and an fp32 sum near 150 is only resolved to ~1e-5 absolute."""
    actual = np.asarray(actual)
    assert actual.shape == expected.shape
    scale = max(1.0, float(np.abs(expected).max()))
    assert np.abs(actual - expected).max() <= tol * scale, np.abs(actual - expected).max()


def test_cuda_q80_linear_matches_cpu(cq, g):
    # test_cuda.cc:679-710 (1-D x, then 2-D x + bias), max-abs tol 1e-4
    blocks = g["tc_q8_0_blocks"]
    expect_near(cq.cudaQ80Linear(g["tc_x"], blocks, [4, 32]), g["tc_q8_0_y"], 1e-4)
    cpu2 = g["tc_q8_0_y2"] + g["tc_bias"][None, :]
    expect_near(cq.cudaQ80Linear(g["tc_x2"], blocks, [4, 32], g["tc_bias"]), cpu2, 1e-4)


def test_cuda_q40_linear_matches_cpu(cq, g):
    # test_cuda.cc:712-728
    expect_near(cq.cudaQ40Linear(g["tc_x"], g["tc_q4_0_blocks"], [4, 32]), g["tc_q4_0_y"], 1e-4)


def test_cuda_q41_linear_matches_cpu(cq, g):
    # test_cuda.cc:730-743 (hand-built q4_1 blocks, makeQ41Blocks)
    expect_near(cq.cudaQ41Linear(g["tc_x"], g["tc_q4_1_blocks"], [4, 32]), g["tc_q4_1_y"], 1e-4)


def test_cuda_quant_device_variants(cq, g):
    # test_cuda.cc:745-774: host / device-weight / device-input agree to 1e-5
    blocks = g["tc_q8_0_blocks"]
    host = cq.cudaQ80Linear(g["tc_x"], blocks, [4, 32])
    w_dev = torch.from_numpy(blocks).cuda()
    dev_weight = cq.cudaQ80LinearDeviceWeight(g["tc_x"], w_dev, 4, [4, 32], None)
    expect_near(dev_weight, host, 1e-5)
    x_dev = torch.from_numpy(g["tc_x"]).cuda()
    dev_input = cq.cudaQ80LinearDeviceInput(x_dev, w_dev, 4, [4, 32], 0)
    assert tuple(dev_input.shape) == (4,)
    expect_near(dev_input.cpu().numpy(), host, 1e-5)


def test_cuda_quant_validation(cq, g):
    # test_cuda.cc:776-809
    blocks = g["tc_q8_0_blocks"]
    with pytest.raises(RuntimeError):
        cq.cudaQ80Linear(np.zeros(16, np.float32), blocks, [4, 32])          # in_features mismatch
    with pytest.raises(RuntimeError):
        cq.cudaQ80Linear(np.zeros(32, np.float32), blocks[:-34], [4, 32])    # short block vector
    with pytest.raises(RuntimeError):
        cq.cudaQ80LinearDeviceWeight(np.zeros(32, np.float32), None, 4, [4, 32], None)  # null
    with pytest.raises(RuntimeError):
        cq.cudaQ80Linear(np.zeros((1, 1, 32), np.float32), blocks, [4, 32])  # rank-3 x


def test_device_input_on_other_device_rejected(cq, g):
    # cuda_quant.cu:342-345: x on a different device than device_id
    x_dev = torch.from_numpy(g["tc_x"]).cuda()
    w_dev = torch.from_numpy(g["tc_q8_0_blocks"]).cuda()
    with pytest.raises(RuntimeError):
        cq.cudaQ80LinearDeviceInput(x_dev, w_dev, 4, [4, 32], 1)


def test_all_formats_golden_shapes(cq, g):
    """Every golden case of make_golden.py through the host-weight entry point."""
    fns = {"q8_0": cq.cudaQ80Linear, "q4_0": cq.cudaQ40Linear, "q4_1": cq.cudaQ41Linear}
    for fmt, fn in fns.items():
        for rows, cols in [(4, 32), (7, 100), (3, 96), (8, 1024), (5, 1), (2, 33), (6, 64)]:
            key = f"{fmt}_{rows}x{cols}"
            for xr in (0, 3):
                y = fn(g[f"{key}_x{xr}"], g[f"{key}_blocks"], [rows, cols])
                ref = g[f"{key}_y{xr}"]
                err = np.linalg.norm(np.atleast_2d(y - ref), axis=1) / np.maximum(
                    np.linalg.norm(np.atleast_2d(ref), axis=1), 1e-30)
                assert err.max() <= 1e-3, (key, xr, err.max())
