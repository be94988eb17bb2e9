"""mlq_linear_swiglu and mlq_linear_bias (include/mlq.h) on the GPU.

* SwiGLU pair: h = silu(x Wg^T) * (x Wu^T) against the oracle (oracle
  linear per matrix, then orc_swiglu, which is bit-exact with the
  reference's swiGlu), relative L2 <= 1e-3 per output row (the linear
  contract), over every route a call can take: the one-token integer GEMV,
  the fp32 GEMV passes (2..8 rows; 13 rows where the GEMM does not take the
  row pitch), the tensor-core GEMM (from 9 rows, or 5 on a large matrix), the
  1-D bulk-copy stream (row pitch not a multiple of 16 B), the any-alignment
  fallback, the dynamic row-tile queue and a captured CUDA graph.  The fused
  launch is also checked against the unfused library calls (mlq_linear per
  matrix, then the oracle's swiglu) at 1e-5.
* Bias: y = x W^T + bias.  The add is one fp32 add in the store, after the
  same sum as mlq_linear's, so it must equal mlq_linear's y + bias bit for
  bit on every route, and the oracle's linear + bias within the contract.
"""
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


def pair_case(oracle, pkg, fmt, out_f, in_f, rows, seed):
    wg = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=seed, std=0.02))
    wu = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=seed + 1, std=0.02))
    x = pkg.synth.normal((rows, in_f), seed=seed + 2, std=1.0)
    return wg, wu, x


def oracle_h(oracle, fmt, x, wg, wu, out_f):
    return oracle.swiglu(oracle.linear(fmt, x, wg, out_f), oracle.linear(fmt, x, wu, out_f))


# (fmt, out, in, rows): one token (integer mode), fp32 passes, GEMM (13 and 16+
# rows, and 8 rows of a large matrix below), partial tiles,
# the 1-D bulk stream (q4_0 in=320: 180-byte rows), the generic fallback (q8_0
# in=96: odd block count per row)
PAIR_CASES = [
    ("q4_0", 1024, 2048, 1),
    ("q8_0", 1000, 1024, 1),
    ("q4_1", 776, 1024, 1),
    ("q4_0", 512, 3584, 2),
    ("q8_0", 300, 2048, 3),
    ("q4_1", 520, 1024, 4),
    ("q4_0", 264, 1024, 8),
    ("q8_0", 256, 1024, 13),
    ("q4_0", 512, 4096, 16),
    ("q4_1", 384, 1024, 64),
    ("q8_0", 300, 1280, 40),
    ("q4_0", 200, 320, 1),
    ("q4_0", 200, 320, 5),
    ("q4_0", 200, 320, 13),      # no GEMM for this row pitch: GEMV passes of 8 + 5 rows
    ("q8_0", 100, 96, 1),
    ("q8_0", 100, 96, 20),
    ("q4_1", 8192, 4096, 8),     # large (2^25 weights): the GEMM pair from 5 rows
]


@pytest.mark.parametrize("fmt,out_f,in_f,rows", PAIR_CASES)
def test_swiglu_pair_matches_oracle(oracle, pkg, fmt, out_f, in_f, rows):
    wg, wu, x = pair_case(oracle, pkg, fmt, out_f, in_f, rows, seed=out_f + 7 * rows)
    xd = dev(x)
    h = pkg.mlq.linear_swiglu(fmt, dev(wg), dev(wu), out_f, in_f, xd).cpu().numpy()
    ref = oracle_h(oracle, fmt, x, wg, wu, out_f)
    assert rel_l2_rows(h, ref).max() <= 1e-3
    # the unfused library path: two linears, then the SwiGLU on the host
    g = pkg.mlq.linear(fmt, dev(wg), out_f, in_f, xd).cpu().numpy()
    u = pkg.mlq.linear(fmt, dev(wu), out_f, in_f, xd).cpu().numpy()
    assert rel_l2_rows(h, oracle.swiglu(g, u)).max() <= 1e-5
    assert pkg.mlq.device_error(0) == 0


def test_swiglu_one_token_vector_x(oracle, pkg):
    """1-D x (the reference's decode shape) gives a 1-D h."""
    fmt, out_f, in_f = "q4_0", 640, 1024
    wg, wu, x = pair_case(oracle, pkg, fmt, out_f, in_f, 1, seed=90)
    h = pkg.mlq.linear_swiglu(fmt, dev(wg), dev(wu), out_f, in_f, dev(x[0]))
    assert tuple(h.shape) == (out_f,)
    ref = oracle_h(oracle, fmt, x[0], wg, wu, out_f)
    assert rel_l2_rows(h.cpu().numpy()[None], ref[None]).max() <= 1e-3


def test_swiglu_dynamic_queue_and_graph(oracle, pkg):
    """A pair with >= 8 row tiles per CTA takes the dynamic row-tile queue
    eagerly; captured in a CUDA graph it runs static row ranges.  Both agree
    with the oracle, and replays of the graph repeat the eager h."""
    fmt, out_f, in_f = "q4_0", 40000, 1024
    wg, wu, x = pair_case(oracle, pkg, fmt, out_f, in_f, 1, seed=91)
    wgd, wud, xd = dev(wg), dev(wu), dev(x)
    eager = pkg.mlq.linear_swiglu(fmt, wgd, wud, out_f, in_f, xd)
    ref = oracle_h(oracle, fmt, x, wg, wu, out_f)
    assert rel_l2_rows(eager.cpu().numpy(), ref).max() <= 1e-3
    h = torch.empty_like(eager)
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        pkg.mlq.linear_swiglu(fmt, wgd, wud, out_f, in_f, xd, h, stream=s)
        s.synchronize()
        g.capture_begin()
        pkg.mlq.linear_swiglu(fmt, wgd, wud, out_f, in_f, xd, h, stream=s)
        g.capture_end()
    h.fill_(0.0)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert rel_l2_rows(h.cpu().numpy(), eager.cpu().numpy()).max() <= 1e-6
    assert pkg.mlq.device_error(0) == 0


def test_swiglu_unaligned_up_falls_back(oracle, pkg):
    """An up matrix that is not 16-B aligned sends the pair to the
    any-alignment path; results still match the oracle."""
    fmt, out_f, in_f = "q4_0", 128, 1024
    wg, wu, x = pair_case(oracle, pkg, fmt, out_f, in_f, 1, seed=92)
    buf = torch.zeros(wu.size + 16, dtype=torch.uint8, device="cuda")
    wu_d = buf[2:2 + wu.size]
    wu_d.copy_(dev(wu))
    h = pkg.mlq.linear_swiglu(fmt, dev(wg), wu_d, out_f, in_f, dev(x)).cpu().numpy()
    assert rel_l2_rows(h, oracle_h(oracle, fmt, x, wg, wu, out_f)).max() <= 1e-3


# (fmt, out, in, rows): integer GEMV, fp32 GEMV, GEMM, 1-D bulk stream, generic
BIAS_CASES = [
    ("q4_0", 4608, 3584, 1),
    ("q8_0", 1000, 1024, 4),
    ("q4_1", 776, 1024, 8),
    ("q4_0", 512, 4096, 16),
    ("q8_0", 384, 1280, 130),
    ("q4_0", 200, 320, 1),
    ("q8_0", 100, 96, 3),
]


@pytest.mark.parametrize("fmt,out_f,in_f,rows", BIAS_CASES)
def test_bias_is_one_add_after_the_sum(oracle, pkg, fmt, out_f, in_f, rows):
    w = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=out_f + rows, std=0.02))
    x = pkg.synth.normal((rows, in_f), seed=rows + 3)
    bias = pkg.synth.normal((out_f,), seed=out_f, std=0.5)
    wd, xd, bd = dev(w), dev(x), dev(bias)
    y = pkg.mlq.linear_bias(fmt, wd, out_f, in_f, xd, bd)
    y0 = pkg.mlq.linear(fmt, wd, out_f, in_f, xd)
    assert torch.equal(y, y0 + bd[None, :])  # bit for bit: the same fp32 add
    ref = oracle.add_bias(oracle.linear(fmt, x, w, out_f), bias)
    assert rel_l2_rows(y.cpu().numpy(), ref).max() <= 1e-3
    yn = pkg.mlq.linear_bias(fmt, wd, out_f, in_f, xd, None)  # null bias = mlq_linear
    assert torch.equal(yn, y0)
    assert pkg.mlq.device_error(0) == 0


def test_reference_bias_case(oracle, pkg, golden_tc):
    """The reference GPU test's fillLinear weights, x and bias
    (tests/test_cuda.cc:66-77, 679-743) through the device bias."""
    g = golden_tc
    for fmt in ("q8_0", "q4_0"):
        y = pkg.mlq.linear_bias(fmt, dev(g[f"tc_{fmt}_blocks"]), 4, 32, dev(g["tc_x2"]), dev(g["tc_bias"]))
        ref = (g[f"tc_{fmt}_y2"] + g["tc_bias"][None, :]).astype(np.float32)
        np.testing.assert_allclose(y.cpu().numpy(), ref, rtol=0, atol=1e-4)


@pytest.fixture(scope="module")
def golden_tc():
    from pathlib import Path
    return np.load(Path(__file__).resolve().parent / "golden" / "reference_quant.npz")
