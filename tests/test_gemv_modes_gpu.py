"""The streaming GEMV's one-token (integer) mode and its scheduling paths.

* Activation edge cases of the integer mode (x carried as int8 slices per
  32-value block): zeros, NaN/Inf propagation, and a block mixing values six
  orders of magnitude apart, against the oracle (the reference's fp32 sums).
* The dynamic row-tile queue (launches with >= 8 row tiles per CTA take row
  tiles from a per-launch queue; each stream has a ring of 32 slots in a
  static array, each slot reset by its launch's last CTA): 600 launches in a
  row wrap a ring many times and must keep giving the same y; two streams
  with a stalled launch, and more streams than rings, must too; a captured
  CUDA graph (static row ranges) must agree with the eager launches.
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


def weights(oracle, pkg, fmt, out_f, in_f, seed):
    return oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=seed, std=0.02))


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
def test_integer_mode_zero_x(oracle, pkg, fmt):
    out_f, in_f = 512, 2048
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 1)
    y = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, torch.zeros(in_f, device="cuda")).cpu().numpy()
    np.testing.assert_array_equal(y, np.zeros(out_f, np.float32))


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
def test_integer_mode_wide_dynamic_range(oracle, pkg, fmt):
    """One value per block 1e3 and the rest ~1e-3: every output vector still
    within the contract of the reference's fp32 sum."""
    out_f, in_f = 384, 4096
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 2)
    x = pkg.synth.normal((1, in_f), seed=3, std=1e-3)
    x[0, ::32] = 1e3 * np.sign(x[0, ::32] + 1e-12)
    y = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, dev(x)).cpu().numpy()
    ref = oracle.linear(fmt, x, blocks, out_f)
    assert rel_l2_rows(y, ref).max() <= 1e-3


@pytest.mark.parametrize("bad", [np.nan, np.inf])
def test_integer_mode_non_finite_x_propagates(oracle, pkg, bad):
    """A NaN or Inf in x makes every output non-finite, as in the reference's
    fp32 sum (every row has a non-zero weight in that block here)."""
    fmt, out_f, in_f = "q8_0", 256, 1024
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 4)
    x = pkg.synth.normal((1, in_f), seed=5)
    x[0, 100] = bad
    y = pkg.mlq.linear(fmt, dev(blocks), out_f, in_f, dev(x)).cpu().numpy()
    ref = oracle.linear(fmt, x, blocks, out_f)
    assert not np.isfinite(ref).any()
    assert not np.isfinite(y).any()


def test_dynamic_tile_queue_survives_ring_wrap(oracle, pkg):
    """A matrix with >= 8 row tiles per CTA (dynamic queue) launched 600 times
    in a row: the stream's ring of 32 slots wraps many times; every y equals
    the first."""
    fmt, out_f, in_f = "q4_0", 80000, 1024
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 6)
    w = dev(blocks)
    x = dev(pkg.synth.normal((1, in_f), seed=7))
    first = pkg.mlq.linear(fmt, w, out_f, in_f, x)
    ref = oracle.linear(fmt, pkg.synth.normal((1, in_f), seed=7)[:, :], blocks, out_f)
    assert rel_l2_rows(first.cpu().numpy(), ref).max() <= 1e-3
    y = torch.empty_like(first)
    mismatches = 0
    for i in range(600):
        y.fill_(float("nan"))
        pkg.mlq.linear(fmt, w, out_f, in_f, x, y)
        if i % 50 == 49 or i == 599:
            torch.cuda.synchronize()
            mismatches += int((y != first).sum())
    assert mismatches == 0
    assert pkg.mlq.device_error(0) == 0


def test_graph_capture_matches_eager(oracle, pkg):
    """Launches captured into a CUDA graph (static row ranges: a graph would
    replay one queue slot) give the same y as eager launches (queue)."""
    fmt, out_f, in_f = "q4_0", 80000, 1024
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 8)
    w = dev(blocks)
    x = dev(pkg.synth.normal((1, in_f), seed=9))
    eager = pkg.mlq.linear(fmt, w, out_f, in_f, x)
    torch.cuda.synchronize()
    y = torch.empty_like(eager)
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        pkg.mlq.linear(fmt, w, out_f, in_f, x, y, stream=s)  # warm-up outside capture
        s.synchronize()
        g.capture_begin()
        pkg.mlq.linear(fmt, w, out_f, in_f, x, y, stream=s)
        g.capture_end()
    y.fill_(0.0)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert rel_l2_rows(y.cpu().numpy(), eager.cpu().numpy()).max() <= 1e-6
    assert pkg.mlq.device_error(0) == 0


def test_tile_queues_two_streams_and_a_stalled_launch(oracle, pkg):
    """Stream A: a sharded launch whose peer never signals (it sits in its
    2 s bounded wait, then reports code 4) followed by 40 queued launches;
    stream B: 300 queued launches issued in between, which run while A is
    stalled.  Each stream takes its own ring of tile-queue slots, so no
    launch shares a slot with one that may run at the same time.  Every y
    must equal the first eager result; after mlq_device_error (which resets
    the queues) 100 more launches on a third stream must too."""
    mlq = pkg.mlq
    fmt, out_f, in_f = "q4_0", 80000, 1024
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 10)
    w = dev(blocks)
    x = dev(pkg.synth.normal((1, in_f), seed=11))
    first = mlq.linear(fmt, w, out_f, in_f, x)
    torch.cuda.synchronize()
    ref = oracle.linear(fmt, pkg.synth.normal((1, in_f), seed=11), blocks, out_f)
    assert rel_l2_rows(first.cpu().numpy(), ref).max() <= 1e-3
    # the stalled sharded launch: rank 0 of two, rows [0, out_f) of a 2*out_f matrix
    big = 2 * out_f
    ys = [torch.zeros((1, big), dtype=torch.float32, device="cuda") for _ in range(2)]
    flags = [torch.zeros(mlq.flag_bytes() // 4, dtype=torch.int32, device="cuda") for _ in range(2)]
    sa, sb = torch.cuda.Stream(), torch.cuda.Stream()
    ya = [torch.empty_like(first) for _ in range(40)]
    yb = [torch.empty_like(first) for _ in range(300)]
    for y in ya + yb:
        y.fill_(float("nan"))
    torch.cuda.synchronize()
    mlq.linear_allgather(fmt, w.data_ptr(), blocks.size // 18, big, in_f, 0, out_f, x.data_ptr(), 1,
                         [y.data_ptr() for y in ys], [f.data_ptr() for f in flags], 0, 1, sa.cuda_stream)
    for i in range(300):
        mlq.linear(fmt, w, out_f, in_f, x, yb[i], stream=sb)
        if i % 7 == 6 and i // 7 < 40:  # the 40 launches of stream A, spread over B's 300
            mlq.linear(fmt, w, out_f, in_f, x, ya[i // 7], stream=sa)
    torch.cuda.synchronize()
    assert mlq.device_error(0) == 4  # the stalled launch gave up; the queues are reset
    bad = [i for i, y in enumerate(yb) if not torch.equal(y, first)]
    bad += [1000 + i for i, y in enumerate(ya) if not torch.equal(y, first)]
    assert not bad, bad[:10]
    sc = torch.cuda.Stream()
    y = torch.empty_like(first)
    for _ in range(100):
        y.fill_(float("nan"))
        mlq.linear(fmt, w, out_f, in_f, x, y, stream=sc)
    torch.cuda.synchronize()
    assert torch.equal(y, first)
    assert mlq.device_error(0) == 0


def test_more_streams_than_rings(oracle, pkg):
    """Streams beyond the 64 tile-queue rings of a device launch with static
    row ranges: 70 streams, one launch each, all equal to the first y."""
    mlq = pkg.mlq
    fmt, out_f, in_f = "q4_0", 80000, 1024
    blocks = weights(oracle, pkg, fmt, out_f, in_f, 12)
    w = dev(blocks)
    x = dev(pkg.synth.normal((1, in_f), seed=13))
    first = mlq.linear(fmt, w, out_f, in_f, x)
    streams = [torch.cuda.Stream() for _ in range(70)]
    ys = [torch.full_like(first, float("nan")) for _ in streams]
    torch.cuda.synchronize()
    for s, y in zip(streams, ys):
        mlq.linear(fmt, w, out_f, in_f, x, y, stream=s)
    torch.cuda.synchronize()
    assert all(torch.equal(y, first) for y in ys)
    assert mlq.device_error(0) == 0
