"""mlq_linear_batch / mlq_linear_batch_host (include/mlq.h) on the GPU.

A batch launches the same kernels as the single-op entry points, in list
order on one stream, so every op's output must equal the single call's bit
for bit; and the oracle (the reference's fp32 sums) within the contract's
relative L2 1e-3 per output vector.  The host form moves x and y itself
and synchronises once; its y must equal the device batch's."""
from __future__ import annotations

import ctypes

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


def _case(pkg, oracle):
    """Ops of one decode step: plain (integer-mode GEMV), bias, SwiGLU pair,
    a 16-row GEMM, a 3-row fp32-mode GEMV and a gathered op in a world of
    one; the matching single calls' outputs; the oracle's."""
    mlq = pkg.mlq
    specs = [("plain", "q4_0", 1000, 3584, 1), ("bias", "q8_0", 512, 1024, 1),
             ("pair", "q4_1", 700, 2048, 1), ("gemm", "q8_0", 384, 1024, 16),
             ("fp32", "q4_0", 640, 2048, 3), ("gather", "q4_0", 2048, 1024, 1)]
    keep, ops, singles, refs, outs = [], [], [], [], []
    for k, (kind, fmt, out_f, in_f, rows) in enumerate(specs):
        wb = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=500 + k, std=0.02))
        x = pkg.synth.normal((rows, in_f), seed=600 + k)
        w, xd = dev(wb), dev(x)
        y = torch.full((rows, out_f), float("nan"), device="cuda")
        keep += [w, xd, y]
        if kind == "pair":
            ub = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=700 + k, std=0.02))
            u = dev(ub)
            keep.append(u)
            ops.append(mlq.linear_op(fmt, w.data_ptr(), out_f, in_f, xd.data_ptr(), rows, y.data_ptr(),
                                     w_up_ptr=u.data_ptr()))
            singles.append(mlq.linear_swiglu(fmt, w, u, out_f, in_f, xd))
            g = oracle.linear(fmt, x, wb, out_f)
            refs.append(oracle.swiglu(g, oracle.linear(fmt, x, ub, out_f)))
        elif kind == "bias":
            b = pkg.synth.normal((out_f,), seed=800 + k, std=0.5)
            bd = dev(b)
            keep.append(bd)
            ops.append(mlq.linear_op(fmt, w.data_ptr(), out_f, in_f, xd.data_ptr(), rows, y.data_ptr(),
                                     bias_ptr=bd.data_ptr()))
            singles.append(mlq.linear_bias(fmt, w, out_f, in_f, xd, bd))
            refs.append(oracle.linear(fmt, x, wb, out_f) + b[None, :])
        elif kind == "gather":
            flags = torch.zeros(mlq.flag_bytes() // 4, dtype=torch.int32, device="cuda")
            keep.append(flags)
            g = mlq.make_gather(1, 0, 0, out_f, [y.data_ptr()], [flags.data_ptr()], epoch=1)
            keep.append(g)
            ops.append(mlq.linear_op(fmt, w.data_ptr(), out_f, in_f, xd.data_ptr(), rows, y.data_ptr(),
                                     gather=g))
            singles.append(mlq.linear(fmt, w, out_f, in_f, xd))
            refs.append(oracle.linear(fmt, x, wb, out_f))
        else:
            ops.append(mlq.linear_op(fmt, w.data_ptr(), out_f, in_f, xd.data_ptr(), rows, y.data_ptr()))
            singles.append(mlq.linear(fmt, w, out_f, in_f, xd))
            refs.append(oracle.linear(fmt, x, wb, out_f))
        outs.append(y)
    return specs, keep, ops, singles, refs, outs


def test_batch_equals_single_calls(pkg, oracle):
    specs, keep, ops, singles, refs, outs = _case(pkg, oracle)
    pkg.mlq.Batch(ops).run(None)
    torch.cuda.synchronize()
    for (kind, *_), y, one, ref in zip(specs, outs, singles, refs):
        yn = y.cpu().numpy()
        np.testing.assert_array_equal(yn, one.cpu().numpy(), err_msg=kind)
        assert rel_l2_rows(yn, ref).max() <= TOL, kind
    assert pkg.mlq.device_error(0) == 0


def test_batch_host_equals_device_batch(pkg, oracle):
    """Host x / host y (pinned), one synchronisation per batch, run twice
    (the second call reuses the staging and, for the gathered op, the next
    epoch)."""
    mlq = pkg.mlq
    specs, keep, ops, singles, refs, outs = _case(pkg, oracle)
    hx, hy = [], []
    host_ops = []
    for op, (kind, fmt, out_f, in_f, rows) in zip(ops, specs):
        x = torch.empty((rows, in_f), dtype=torch.float32).pin_memory()
        y = torch.full((rows, out_f), float("nan"), dtype=torch.float32).pin_memory()
        hx.append(x)
        hy.append(y)
        h = mlq.LinearOp.from_buffer_copy(op)
        h.x, h.y = x.data_ptr(), y.data_ptr()
        host_ops.append(h)
    batch = mlq.Batch(host_ops)
    for it in range(2):
        for k, (kind, fmt, out_f, in_f, rows) in enumerate(specs):
            hx[k].copy_(torch.from_numpy(pkg.synth.normal((rows, in_f), seed=900 + 10 * it + k)))
            hy[k].fill_(float("nan"))
        if it == 1:
            keep[[i for i, o in enumerate(keep) if isinstance(o, mlq.Gather)][0]].epoch = 2
        batch.run_host(0)
        for k, (kind, fmt, out_f, in_f, rows) in enumerate(specs):
            # the device batch on the same x gives the same y, bit for bit
            xd = hx[k].cuda()
            op = mlq.LinearOp.from_buffer_copy(ops[k])
            op.x = xd.data_ptr()
            if kind == "gather":
                op.gather = None  # compare with a plain call on one GPU
            yd = torch.empty((rows, out_f), device="cuda")
            op.y = yd.data_ptr()
            mlq.Batch([op]).run(None)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(hy[k].numpy(), yd.cpu().numpy(), err_msg=f"{kind} call {it}")
    assert mlq.device_error(0) == 0


@pytest.mark.parametrize("rows", [4, 16])
def test_batch_groups_ops_sharing_x(pkg, oracle, rows):
    """Consecutive ops that read one x and take the batched-decode GEMM run
    as one grouped launch (Q, K, V of a layer; up to four matrices): each
    op's y within the contract of the oracle and within 1e-5 of the op run
    alone (a grouped launch splits the work at other points, so the fp32
    sums of split row tiles may round differently).  The op list: q, k, v
    (one with a bias) on x0, a matrix on x1 (ends the group), five matrices
    on x2 (a group of four, then one), and a SwiGLU pair on x2 (its own
    group of two)."""
    mlq = pkg.mlq
    fmt, in_f = "q8_0", 2048
    specs = [(0, 1024), (0, 256), (0, 256), (1, 640), (2, 300), (2, 128), (2, 1000), (2, 512), (2, 384)]
    xs = [pkg.synth.normal((rows, in_f), seed=900 + k) for k in range(3)]
    xd = [dev(x) for x in xs]
    keep, ops, refs, singles, outs = [], [], [], [], []
    for k, (xi, out_f) in enumerate(specs):
        wb = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=950 + k, std=0.02))
        w = dev(wb)
        y = torch.full((rows, out_f), float("nan"), device="cuda")
        keep.append(w)
        outs.append(y)
        assert mlq.takes_bgemm(rows, out_f, in_f)
        ref = oracle.linear(fmt, xs[xi], wb, out_f)
        if k == 1:
            b = pkg.synth.normal((out_f,), seed=990, std=0.5)
            bd = dev(b)
            keep.append(bd)
            ops.append(mlq.linear_op(fmt, w.data_ptr(), out_f, in_f, xd[xi].data_ptr(), rows, y.data_ptr(),
                                     bias_ptr=bd.data_ptr()))
            singles.append(mlq.linear_bias(fmt, w, out_f, in_f, xd[xi], bd))
            ref = ref + b[None, :]
        else:
            ops.append(mlq.linear_op(fmt, w.data_ptr(), out_f, in_f, xd[xi].data_ptr(), rows, y.data_ptr()))
            singles.append(mlq.linear(fmt, w, out_f, in_f, xd[xi]))
        refs.append(ref)
    gb = oracle.quantize(fmt, pkg.synth.normal((700, in_f), seed=991, std=0.02))
    ub = oracle.quantize(fmt, pkg.synth.normal((700, in_f), seed=992, std=0.02))
    g, u = dev(gb), dev(ub)
    h = torch.full((rows, 700), float("nan"), device="cuda")
    keep += [g, u, h]
    ops.append(mlq.linear_op(fmt, g.data_ptr(), 700, in_f, xd[2].data_ptr(), rows, h.data_ptr(),
                             w_up_ptr=u.data_ptr()))
    refs.append(oracle.swiglu(oracle.linear(fmt, xs[2], gb, 700), oracle.linear(fmt, xs[2], ub, 700)))
    singles.append(None)
    outs.append(h)
    mlq.Batch(ops).run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    for k, (y, ref, single) in enumerate(zip(outs, refs, singles)):
        yn = y.cpu().numpy()
        assert rel_l2_rows(yn, ref).max() <= TOL, k
        if single is not None:
            assert rel_l2_rows(yn, single.cpu().numpy()).max() <= 1e-5, k
    assert mlq.device_error(0) == 0


def test_batch_gemv_runs_respect_dependencies(pkg, oracle):
    """One-token ops that do not touch one another's outputs run back to
    back without waiting for each other; an op that reads an earlier op's y
    (a chain) or overwrites an earlier op's x must still see, or leave, the
    right data.  Ops: y1 = W1 x0; y2 = W2 y1 (reads y1); y3 = W3 x3;
    y4 = W4 x4; then W5 x3 written into x4's buffer (after op 4 read it)."""
    mlq = pkg.mlq
    fmt = "q4_0"
    n = 1024
    ws, keep = [], []
    for k in range(5):
        wb = oracle.quantize(fmt, pkg.synth.normal((n, n), seed=1100 + k, std=0.02))
        ws.append((wb, dev(wb)))
    x0 = pkg.synth.normal((1, n), seed=1200)
    x3 = pkg.synth.normal((1, n), seed=1201)
    x4 = pkg.synth.normal((1, n), seed=1202)
    x0d, x3d, x4d = dev(x0), dev(x3), dev(x4)
    y1 = torch.full((1, n), float("nan"), device="cuda")
    y2 = torch.full((1, n), float("nan"), device="cuda")
    y3 = torch.full((1, n), float("nan"), device="cuda")
    y4 = torch.full((1, n), float("nan"), device="cuda")
    ops = [mlq.linear_op(fmt, ws[0][1].data_ptr(), n, n, x0d.data_ptr(), 1, y1.data_ptr()),
           mlq.linear_op(fmt, ws[1][1].data_ptr(), n, n, y1.data_ptr(), 1, y2.data_ptr()),   # reads y1
           mlq.linear_op(fmt, ws[2][1].data_ptr(), n, n, x3d.data_ptr(), 1, y3.data_ptr()),
           mlq.linear_op(fmt, ws[3][1].data_ptr(), n, n, x4d.data_ptr(), 1, y4.data_ptr()),
           mlq.linear_op(fmt, ws[4][1].data_ptr(), n, n, x3d.data_ptr(), 1, x4d.data_ptr())]  # overwrites x4 after op 4 read it
    mlq.Batch(ops).run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    r1 = oracle.linear(fmt, x0, ws[0][0], n)
    r2 = oracle.linear(fmt, y1.cpu().numpy(), ws[1][0], n)
    r3 = oracle.linear(fmt, x3, ws[2][0], n)
    r4 = oracle.linear(fmt, x4, ws[3][0], n)
    r5 = oracle.linear(fmt, x3, ws[4][0], n)
    assert rel_l2_rows(y1.cpu().numpy(), r1).max() <= TOL
    assert rel_l2_rows(y2.cpu().numpy(), r2).max() <= TOL
    assert rel_l2_rows(y3.cpu().numpy(), r3).max() <= TOL
    assert rel_l2_rows(y4.cpu().numpy(), r4).max() <= TOL  # op 4 read x4 before op 5 overwrote it
    assert rel_l2_rows(x4d.cpu().numpy(), r5).max() <= TOL
    assert mlq.device_error(0) == 0


def _run_case(pkg, oracle, fmt, shapes, bias_at=(), seed=1300):
    """One-row ops of one format on distinct x and y: the batch runs them as
    one persistent launch per eight ops.  Returns the batch's ops, outputs,
    the matching single calls' outputs and the oracle's."""
    mlq = pkg.mlq
    keep, ops, outs, singles, refs, xds = [], [], [], [], [], []
    for k, (out_f, in_f) in enumerate(shapes):
        wb = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=seed + k, std=0.02))
        x = pkg.synth.normal((1, in_f), seed=seed + 100 + k)
        w, xd = dev(wb), dev(x)
        y = torch.full((1, out_f), float("nan"), device="cuda")
        keep.append(w)
        xds.append(xd)
        ref = oracle.linear(fmt, x, wb, out_f)
        if k in bias_at:
            b = pkg.synth.normal((out_f,), seed=seed + 200 + k, std=0.5)
            bd = dev(b)
            keep.append(bd)
            ops.append(mlq.linear_op(fmt, w.data_ptr(), out_f, in_f, xd.data_ptr(), 1, y.data_ptr(),
                                     bias_ptr=bd.data_ptr()))
            singles.append(mlq.linear_bias(fmt, w, out_f, in_f, xd, bd))
            ref = ref + b[None, :]
        else:
            ops.append(mlq.linear_op(fmt, w.data_ptr(), out_f, in_f, xd.data_ptr(), 1, y.data_ptr()))
            singles.append(mlq.linear(fmt, w, out_f, in_f, xd))
        outs.append(y)
        refs.append(ref)
    return keep, xds, ops, outs, singles, refs


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_1"])
def test_batch_run_of_one_row_ops(pkg, oracle, fmt):
    """A run of independent one-row ops (ten: two persistent launches) with
    mixed shapes -- a long K (10 K-tiles), partial K-tiles, row counts that
    are not tile multiples, a single row, biases -- gives every op's y bit
    for bit as the op run alone (the same integer-mode decode and summation
    order), and within the contract of the oracle."""
    shapes = [(1000, 3584), (4096, 18944), (1, 1024), (333, 2048), (2500, 4096), (64, 1280),
              (700, 3584), (129, 5120), (4100, 1024), (90, 2304)]
    keep, xds, ops, outs, singles, refs = _run_case(pkg, oracle, fmt, shapes, bias_at=(1, 4, 9))
    pkg.mlq.Batch(ops).run(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    for k, (y, one, ref) in enumerate(zip(outs, singles, refs)):
        yn = y.cpu().numpy()
        np.testing.assert_array_equal(yn, one.cpu().numpy(), err_msg=f"op {k} {shapes[k]}")
        assert rel_l2_rows(yn, ref).max() <= TOL, k
    assert pkg.mlq.device_error(0) == 0


def test_batch_run_in_a_cuda_graph(pkg, oracle):
    """The same run captured in a CUDA graph (no tile queue while capturing:
    each CTA takes a fixed stride of row tiles) and replayed twice on new x
    values: every y equal to the op run alone."""
    mlq = pkg.mlq
    fmt = "q4_0"
    shapes = [(3584, 3584), (512, 3584), (18944, 3584), (3584, 18944)]
    keep, xds, ops, outs, singles, refs = _run_case(pkg, oracle, fmt, shapes, bias_at=(1,), seed=1500)
    batch = mlq.Batch(ops)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        batch.run(s.cuda_stream)  # sizes the stream's workspace before the capture
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        batch.run(s.cuda_stream)
    for it in range(2):
        for k, x in enumerate(xds):
            x.copy_(torch.from_numpy(pkg.synth.normal(tuple(x.shape), seed=1600 + 10 * it + k)))
        for y in outs:
            y.fill_(float("nan"))
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        for k, ((out_f, in_f), y, op) in enumerate(zip(shapes, outs, ops)):
            one = mlq.LinearOp.from_buffer_copy(op)
            yd = torch.empty((1, out_f), device="cuda")
            one.y = yd.data_ptr()
            mlq.Batch([one]).run(None)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(y.cpu().numpy(), yd.cpu().numpy(), err_msg=f"replay {it} op {k}")
    del g
    assert mlq.device_error(0) == 0


def test_batch_run_with_gathered_ops_in_a_world_of_one(pkg, oracle):
    """Gathered one-row ops (a world of one; one with a deferred wait, one
    with a bias) join a run with plain ops: every y bit for bit as the op
    run alone, and within the contract of the oracle."""
    mlq = pkg.mlq
    fmt = "q8_0"
    shapes = [(2048, 4096), (1000, 2048), (4096, 1024), (512, 4096)]
    keep, xds, ops, outs, singles, refs = _run_case(pkg, oracle, fmt, shapes, bias_at=(3,), seed=1700)
    flags = torch.zeros(mlq.flag_bytes() // 4, dtype=torch.int32, device="cuda")
    gathers = []
    for k in (1, 3):
        out_f = shapes[k][0]
        g = mlq.make_gather(1, 0, 0, out_f, [outs[k].data_ptr()], [flags.data_ptr()], epoch=1,
                            defer_wait=(k == 1))
        gathers.append(g)
        op = mlq.LinearOp.from_buffer_copy(ops[k])
        op.gather = ctypes.addressof(g)
        op.block_count = mlq.blocks_per_row(shapes[k][1]) * out_f
        ops[k] = op
    pkg.mlq.Batch(ops).run(torch.cuda.current_stream().cuda_stream)
    mlq.gather_wait(gathers[0], torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    for k, (y, one, ref) in enumerate(zip(outs, singles, refs)):
        yn = y.cpu().numpy()
        np.testing.assert_array_equal(yn, one.cpu().numpy(), err_msg=f"op {k}")
        assert rel_l2_rows(yn, ref).max() <= TOL, k
    assert mlq.device_error(0) == 0


def test_batch_host_overlaps_the_download(pkg, oracle):
    """A host batch whose y download is large (here 401 KB): the largest
    plain one-row op's last rows run as a second launch while the rest of
    y is copied back.  Every y equals the device batch's bit for bit (each
    row's arithmetic is the same), twice in a row, and the big op's rows on
    both sides of the split match the oracle."""
    mlq = pkg.mlq
    specs = [("q8_0", 2048, 4096), ("q4_0", 98304, 1024)]
    keep, dev_ops, host_ops, hx, hy, refs = [], [], [], [], [], []
    for k, (fmt, out_f, in_f) in enumerate(specs):
        wb = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=1800 + k, std=0.02))
        w = dev(wb)
        x = torch.from_numpy(pkg.synth.normal((1, in_f), seed=1900 + k)).pin_memory()
        yh = torch.full((1, out_f), float("nan")).pin_memory()
        xd = x.cuda()
        yd = torch.full((1, out_f), float("nan"), device="cuda")
        keep += [w, xd, yd]
        dev_ops.append(mlq.linear_op(fmt, w.data_ptr(), out_f, in_f, xd.data_ptr(), 1, yd.data_ptr()))
        host_ops.append(mlq.linear_op(fmt, w.data_ptr(), out_f, in_f, x.data_ptr(), 1, yh.data_ptr()))
        hx.append(x)
        hy.append(yh)
        refs.append((wb, yd))
    mlq.Batch(dev_ops).run(None)
    torch.cuda.synchronize()
    hb = mlq.Batch(host_ops)
    for it in range(2):
        for y in hy:
            y.fill_(float("nan"))
        hb.run_host(0)
        for k, (y, (_, yd)) in enumerate(zip(hy, refs)):
            np.testing.assert_array_equal(y.numpy(), yd.cpu().numpy(), err_msg=f"op {k} call {it}")
    # the big op's rows (every 37th, and the last 256: both sides of the
    # split point) against the oracle
    fmt, out_f, in_f = specs[1]
    rows = np.unique(np.r_[0:out_f:37, out_f - 256:out_f])
    wb = refs[1][0].reshape(out_f, -1)[rows]
    ref = oracle.linear(fmt, hx[1].numpy(), wb.reshape(-1), len(rows))
    assert rel_l2_rows(hy[1].numpy()[:, rows], ref).max() <= TOL
    assert mlq.device_error(0) == 0
