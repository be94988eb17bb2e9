"""mlq_linear_noalloc (include/mlq.h) against mlq_linear.

The no-alloc entry point runs the same kernels as mlq_linear; only the
GEMM's x split lives in a static device array instead of a per-stream
workspace.  Each case makes two calls in a row on one stream (the second
reuses the scratch the first one wrote) and checks both against mlq_linear
at relative L2 1e-5 per output row (the contract is 1e-3; the same kernels
should agree to the last bit, unless the scratch is too small for the
GEMM's split-K partials -- see test_noalloc_full_scratch_allocates_nothing).  This file is collected last so that it also
runs after every other GPU test in one process."""
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


def _pair(pkg, oracle, fmt, out_f, in_f, rows, seed):
    blocks = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=seed, std=0.02))
    xs = [dev(pkg.synth.normal((rows, in_f), seed=seed + k + 1)) for k in range(2)]
    return dev(blocks), xs


@pytest.mark.parametrize("fmt,out_f,in_f,rows", [
    ("q4_0", 512, 4096, 128),   # tensor-core GEMM
    ("q8_0", 384, 1280, 200),   # GEMM, partial tiles
    ("q4_1", 300, 1024, 64),
    ("q8_0", 256, 1024, 9),     # GEMM at its smallest row count
    ("q4_0", 256, 2048, 3),     # GEMV (no scratch at all)
])
def test_noalloc_matches_linear_two_calls(pkg, oracle, fmt, out_f, in_f, rows):
    w, xs = _pair(pkg, oracle, fmt, out_f, in_f, rows, seed=out_f + rows)
    ys = [torch.empty((rows, out_f), dtype=torch.float32, device="cuda") for _ in xs]
    for x, y in zip(xs, ys):  # back to back, no synchronisation in between
        pkg.mlq.linear_noalloc(fmt, w, out_f, in_f, x, y)
    refs = [pkg.mlq.linear(fmt, w, out_f, in_f, x) for x in xs]
    torch.cuda.synchronize()
    for y, ref in zip(ys, refs):
        err = rel_l2_rows(y.cpu().numpy(), ref.cpu().numpy()).max()
        assert err <= 1e-5, err
    assert pkg.mlq.device_error(0) == 0


def test_noalloc_full_scratch_allocates_nothing(pkg, oracle):
    """rows * in * 4 == MLQ_NOALLOC_SCRATCH_BYTES exactly, on a fresh stream:
    free device memory is unchanged across two calls (mlq_linear would
    allocate a workspace for a new stream).  The x split fills the scratch,
    so this call runs the GEMM over the whole K extent where mlq_linear
    splits K into ranges (its workspace holds their partial sums): the two
    differ by summation order, checked at the GEMM's 1e-4."""
    fmt, out_f, in_f = "q4_0", 256, 4096
    rows = pkg.mlq.NOALLOC_SCRATCH_BYTES // (4 * in_f)
    w, xs = _pair(pkg, oracle, fmt, out_f, in_f, rows, seed=11)
    ys = [torch.empty((rows, out_f), dtype=torch.float32, device="cuda") for _ in xs]
    pkg.mlq.linear_noalloc(fmt, w, out_f, in_f, xs[0], ys[0])  # one-time setup, kernels loaded
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    free_before = torch.cuda.mem_get_info()[0]
    with torch.cuda.stream(side):
        for x, y in zip(xs, ys):
            pkg.mlq.linear_noalloc(fmt, w, out_f, in_f, x, y)
    torch.cuda.synchronize()
    free_after = torch.cuda.mem_get_info()[0]
    assert free_after == free_before, (free_before, free_after)
    for x, y in zip(xs, ys):
        ref = pkg.mlq.linear(fmt, w, out_f, in_f, x)
        torch.cuda.synchronize()
        assert rel_l2_rows(y.cpu().numpy(), ref.cpu().numpy()).max() <= 1e-4


def test_noalloc_rejects_oversize_gemm(pkg, oracle):
    fmt, out_f, in_f = "q4_0", 128, 4096
    rows = pkg.mlq.NOALLOC_SCRATCH_BYTES // (4 * in_f) + 1
    w, xs = _pair(pkg, oracle, fmt, out_f, in_f, rows, seed=21)
    y = torch.zeros((rows, out_f), dtype=torch.float32, device="cuda")
    with pytest.raises(pkg.mlq.MLQError) as ei:
        pkg.mlq.linear_noalloc(fmt, w, out_f, in_f, xs[0], y)
    assert ei.value.status == 9 and "static scratch" in ei.value.message
    torch.cuda.synchronize()
    assert float(y.abs().max()) == 0.0  # rejected before any launch


def test_noalloc_large_x_below_gemm_rows(pkg, oracle):
    """rows below the GEMM threshold take the GEMV, which needs no scratch:
    x larger than the scratch is accepted and matches mlq_linear."""
    fmt, out_f, in_f = "q8_0", 32, 524352
    rows = pkg.mlq.GEMM_MIN_ROWS - 1
    assert not pkg.mlq.takes_gemm(rows, out_f, in_f)
    assert rows * in_f * 4 > pkg.mlq.NOALLOC_SCRATCH_BYTES
    w, xs = _pair(pkg, oracle, fmt, out_f, in_f, rows, seed=31)
    y = torch.empty((rows, out_f), dtype=torch.float32, device="cuda")
    pkg.mlq.linear_noalloc(fmt, w, out_f, in_f, xs[0], y)
    pkg.mlq.linear_noalloc(fmt, w, out_f, in_f, xs[1], y)
    ref = pkg.mlq.linear(fmt, w, out_f, in_f, xs[1])
    torch.cuda.synchronize()
    assert rel_l2_rows(y.cpu().numpy(), ref.cpu().numpy()).max() <= 1e-5
    assert pkg.mlq.device_error(0) == 0
