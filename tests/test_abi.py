"""CPU tests of the C ABI: the library loads, exports every entry point
include/mlq.h declares, and rejects bad arguments on the host before any
CUDA call (so these run without a GPU)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_symbols():
    names = []
    for h in HEADERS:
        text = h.read_text()
        names += re.findall(r"MLQ_API\s+[\w\s\*]+?\b(mlq_\w+)\s*\(", text)
    return sorted(set(names))


def test_headers_declare_entry_points():
    names = declared_symbols()
    assert "mlq_linear" in names and "mlq_quantize" in names and len(names) >= 10


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.mlq.lib()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_library_facts(pkg):
    lib = pkg.mlq.lib()
    assert lib.mlq_built() == 1
    assert [lib.mlq_block_bytes(f) for f in (8, 2, 3, 0)] == [34, 18, 20, 0]
    assert lib.mlq_block_count(4864, 896) == 4864 * 28
    assert lib.mlq_block_count(3, 100) == 12
    assert lib.mlq_block_count(0, 5) == 0
    assert lib.mlq_status_string(5) == b"block count mismatch"


def _linear_status(pkg, fmt=8, w=0x1000, nb=4, out=4, inf=32, x=0x2000, rows=1, y=0x3000):
    lib = pkg.mlq.lib()
    return lib.mlq_linear(fmt, w, nb, out, inf, x, rows, y, None)


def test_validation_before_any_cuda_call(pkg):
    """The reference's checks (src/cuda_quant.cu:198-227, 305-307); the
    pointers are never dereferenced because validation fails first."""
    mlq = pkg.mlq
    lib = mlq.lib()
    assert _linear_status(pkg, fmt=7) == 1                    # unknown format
    assert _linear_status(pkg, w=None) == 2                   # null weight pointer
    assert b"null weight pointer" in lib.mlq_last_error()
    assert _linear_status(pkg, out=0) == 3                    # empty
    assert b"empty tensors are not supported" in lib.mlq_last_error()
    assert _linear_status(pkg, inf=-1) == 3
    assert _linear_status(pkg, rows=0) == 3
    assert _linear_status(pkg, x=None) == 2
    assert _linear_status(pkg, nb=3) == 5                     # short block vector
    assert b"expected 4, got 3" in lib.mlq_last_error()
    assert _linear_status(pkg, nb=4, inf=33) == 5             # 33 values -> 2 blocks per row
    assert b"expected 8, got 4" in lib.mlq_last_error()
    # (no call here ever passes validation: the pointers above are fake)


def test_fused_entry_points_validate_first(pkg):
    """mlq_linear_bias / mlq_linear_swiglu run mlq_linear's checks, and the
    pair's second weight pointer is checked too, all before any CUDA call."""
    lib = pkg.mlq.lib()
    assert lib.mlq_linear_bias(7, 0x1000, 4, 4, 32, 0x2000, 1, 0x4000, 0x3000, None) == 1
    assert lib.mlq_linear_bias(8, None, 4, 4, 32, 0x2000, 1, 0x4000, 0x3000, None) == 2
    assert lib.mlq_linear_bias(8, 0x1000, 3, 4, 32, 0x2000, 1, 0x4000, 0x3000, None) == 5
    assert b"mlq_linear_bias(Q80)" in lib.mlq_last_error()
    assert lib.mlq_linear_swiglu(2, 0x1000, None, 4, 4, 32, 0x2000, 1, 0x3000, None) == 2
    assert b"null up-projection weight pointer" in lib.mlq_last_error()
    assert lib.mlq_linear_swiglu(2, None, 0x1800, 4, 4, 32, 0x2000, 1, 0x3000, None) == 2
    assert lib.mlq_linear_swiglu(2, 0x1000, 0x1800, 4, 4, 32, 0x2000, 0, 0x3000, None) == 3
    assert lib.mlq_linear_swiglu(2, 0x1000, 0x1800, 4, 4, 32, None, 1, 0x3000, None) == 2
    assert lib.mlq_linear_swiglu(3, 0x1000, 0x1800, 5, 4, 32, 0x2000, 1, 0x3000, None) == 5


def test_host_entry_points_validate_first(pkg):
    mlq = pkg.mlq
    x = np.zeros(32, np.float32)
    with pytest.raises(mlq.MLQError) as e:
        mlq.linear_host_weight("q8_0", np.zeros(3 * 34, np.uint8), 4, 32, x)  # 3 blocks for 4 rows
    assert e.value.status == 5
    with pytest.raises(mlq.MLQError) as e:
        mlq.linear_host("q4_0", 0, 4, 32, x)  # null device weight
    assert e.value.status == 2
    lib = mlq.lib()
    assert lib.mlq_quantize(8, None, 4, 32, None, None) == 2
    assert lib.mlq_quantize(8, 0x1000, 0, 32, 0x2000, None) == 3
    assert lib.mlq_dequantize(2, 0x1000, 5, 4, 32, 0x2000, None) == 5


def test_cuda_quant_shape_errors_raise_runtime_error(pkg):
    """Reference-named entry points raise RuntimeError like the reference
    (tests/test_cuda.cc:776-809): bad in_features, short blocks, null
    weight pointer, rank-3 x -- all caught before the GPU."""
    import importlib
    cq = importlib.import_module("mini_llama_b200.cuda_quant")
    blocks = np.zeros(4 * 34, np.uint8)
    with pytest.raises(RuntimeError):
        cq.cudaQ80Linear(np.zeros(16, np.float32), blocks, [4, 32])
    with pytest.raises(RuntimeError):
        cq.cudaQ80Linear(np.zeros(32, np.float32), blocks[:-34], [4, 32])
    with pytest.raises(RuntimeError):
        cq.cudaQ80LinearDeviceWeight(np.zeros(32, np.float32), None, 4, [4, 32])
    with pytest.raises(RuntimeError):
        cq.cudaQ80Linear(np.zeros((1, 1, 32), np.float32), blocks, [4, 32])


def test_missing_library_fails_loudly(pkg, tmp_path, monkeypatch):
    mlq = pkg.mlq
    monkeypatch.setattr(mlq, "_lib", None)
    monkeypatch.setattr(mlq, "LIB_PATH", tmp_path / "libmlq.so")
    with pytest.raises(FileNotFoundError):
        mlq.lib()


def test_gemm_routing_rule_matches_header(pkg, tmp_path):
    """mlq.takes_gemm (Python) and MLQ_GEMM_ROWS_RULE (include/mlq.h, the rule
    the library compiles) agree on a grid of rows x matrix sizes, and the
    Python constants equal the header's.  The header is plain C: gcc builds
    a probe that prints the macro's answers."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    rows = [1, 2, 4, 5, 8, 9, 15, 16, 512]
    shapes = [(32, 524352), (4608, 3584), (4096, 4096), (8192, 4096), (8191, 4096), (3584, 18944),
              (152064, 3584)]
    src = tmp_path / "rule.c"
    lines = ['#include <stdio.h>', '#include "mlq.h"', "int main(void) {",
             '  printf("%d %d %lld %d %d %d\\n", MLQ_GEMM_MIN_ROWS, MLQ_GEMM_LARGE_MIN_ROWS, '
             "(long long)MLQ_GEMM_LARGE_MIN_WEIGHTS, MLQ_BGEMM_MIN_ROWS, MLQ_BGEMM_MAX_ROWS, "
             "MLQ_BATCH_RUN_MAX_OPS);"]
    for r in rows:
        for o, i in shapes:
            lines.append(f'  printf("%d\\n", (int)(MLQ_GEMM_ROWS_RULE({r}, {o}, {i})));')
    lines.append("  return 0;\n}")
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "rule"
    subprocess.run([gcc, "-std=c99", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    mlq = pkg.mlq
    assert out[0].split() == [str(v) for v in (mlq.GEMM_MIN_ROWS, mlq.GEMM_LARGE_MIN_ROWS, mlq.GEMM_LARGE_MIN_WEIGHTS,
                                               mlq.BGEMM_MIN_ROWS, mlq.BGEMM_MAX_ROWS, mlq.RUN_MAX_OPS)]
    got = [int(v) for v in out[1:] if v.strip()]
    want = [int(mlq.takes_gemm(r, o, i)) for r in rows for o, i in shapes]
    assert got == want


def test_noalloc_range_rule_before_any_cuda_call(pkg):
    """mlq_linear_noalloc rejects, before any CUDA call, exactly the calls
    that take the bf16 tensor-core GEMM (MLQ_GEMM_ROWS_RULE, not taken by the
    batched-decode GEMM) with an x split above the static scratch.
    (Pointers are fake: a rejected call never touches them.)"""
    mlq = pkg.mlq
    lib = mlq.lib()
    scratch = mlq.NOALLOC_SCRATCH_BYTES

    def status(fmt, rows, out_f, in_f, w=0x1000):
        nb = mlq.block_count(out_f, in_f)
        return lib.mlq_linear_noalloc(fmt, w, nb, out_f, in_f, 0x2000, rows, 0x3000, None)

    # 33 rows (above the batched-decode GEMM's 32) whose x split exceeds the
    # scratch; a multiple of 256 values, so q8_0 rows have a 16-B multiple pitch
    in_f = (scratch // (4 * 33) // 256 + 1) * 256
    assert mlq.takes_gemm(33, 32, in_f) and not mlq.takes_bgemm(33, 32, in_f)
    assert status(8, 33, 32, in_f) == 9
    assert b"static scratch" in lib.mlq_last_error()
    # 9 rows with in % 32 == 16 (q4_1, 16-B row pitch): the bf16 GEMM, rejected
    in_q41 = 14568 * 32 - 16
    assert not mlq.takes_bgemm(9, 32, in_q41) and 9 * in_q41 * 4 > scratch
    assert status(3, 9, 32, in_q41) == 9
    # Calls no GEMM with this limit takes stream through the GEMV or run the
    # batched-decode GEMM (which falls back to the GEMV when its scratch does
    # not fit): never MLQ_ERR_RANGE.  These calls pass the host checks and go
    # on to CUDA, so they run only where there is no GPU to reach (the
    # pointers are fake); there the first CUDA call fails with MLQ_ERR_CUDA.
    import torch
    if torch.cuda.is_available():
        return
    assert status(8, 9, 32, in_f) != 9            # batched-decode GEMM rows
    assert status(8, 33, 32, in_f, w=0x1002) != 9  # weights not 16-B aligned
    odd_in = in_f + 4  # in % 8 == 4
    assert odd_in % 8 == 4 and mlq.takes_gemm(33, 32, odd_in)
    assert status(8, 33, 32, odd_in) != 9


def test_batch_structs_match_header(pkg, tmp_path):
    """The ctypes mirrors of mlq_gather / mlq_linear_op have the header's
    field offsets and sizes (a gcc-built probe prints them)."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    mlq = pkg.mlq
    checks = [("mlq_gather", mlq.Gather), ("mlq_linear_op", mlq.LinearOp)]
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "mlq.h"', "int main(void) {"]
    for cname, cls in checks:
        lines.append(f'  printf("%zu\\n", sizeof({cname}));')
        for f, _ in cls._fields_:
            lines.append(f'  printf("%zu\\n", offsetof({cname}, {f}));')
    lines.append("  return 0;\n}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-std=c99", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True,
                                          text=True).stdout.split()]
    want = []
    for _, cls in checks:
        want.append(ctypes.sizeof(cls))
        want += [getattr(cls, f).offset for f, _ in cls._fields_]
    assert got == want


def test_batch_validates_every_op_before_any_cuda_call(pkg):
    """A batch whose third op is bad launches nothing and names that op; the
    host form checks the same things (pointers are fake: nothing runs)."""
    mlq = pkg.mlq
    lib = mlq.lib()
    good = mlq.linear_op("q8_0", 0x1000, 4, 32, 0x2000, 1, 0x3000)
    bad_blocks = mlq.LinearOp(8, 4, 32, 1, 0x1000, None, 3, 0x2000, None, 0x3000, None)
    pair_bias = mlq.linear_op("q4_0", 0x1000, 4, 32, 0x2000, 1, 0x3000, w_up_ptr=0x1800, bias_ptr=0x4000)
    for ops, code, text in [([good, good, bad_blocks], 5, b"op 2"),
                            ([good, pair_bias], 9, b"takes no bias"),
                            ([mlq.linear_op("q4_1", None, 4, 32, 0x2000, 1, 0x3000)], 2, b"op 0")]:
        arr = (mlq.LinearOp * len(ops))(*ops)
        assert lib.mlq_linear_batch(arr, len(ops), None) == code
        assert text in lib.mlq_last_error()
        assert lib.mlq_linear_batch_host(arr, len(ops), 0, None) == code
    assert lib.mlq_linear_batch(None, -1, None) == 3
    assert lib.mlq_linear_batch(None, 0, None) == 0  # an empty batch is a no-op
    # a gathered op: mlq_linear_allgather's checks (epoch 0, a pair)
    g = mlq.make_gather(2, 0, 0, 2, [0x5000, 0x6000], [0x7000, 0x8000], epoch=0)
    op = mlq.linear_op("q4_0", 0x1000, 4, 32, 0x2000, 1, 0x3000, gather=g)
    assert op.block_count == 2  # this rank's two rows
    arr = (mlq.LinearOp * 1)(op)
    assert lib.mlq_linear_batch(arr, 1, None) == 10
    g.epoch = 1
    arr[0].w_up = 0x1800
    assert lib.mlq_linear_batch(arr, 1, None) == 9
    assert b"no up projection" in lib.mlq_last_error()


def test_gather_wait_validates_before_any_cuda_call(pkg):
    """mlq_gather_wait and a deferred gathered op check their arguments on
    the host first (pointers are fake: nothing runs)."""
    mlq = pkg.mlq
    lib = mlq.lib()
    assert lib.mlq_gather_wait(None, None) == 2
    g = mlq.make_gather(2, 2, 0, 4, [0x3000, 0x3100], [0x4000, 0x4100], epoch=1, defer_wait=True)
    assert lib.mlq_gather_wait(ctypes.byref(g), None) == 10  # rank outside the world
    g = mlq.make_gather(2, 1, 0, 4, [0x3000, 0x3100], [0x4000, 0x4100], epoch=0, defer_wait=True)
    assert lib.mlq_gather_wait(ctypes.byref(g), None) == 10  # epoch 0
    assert b"epoch" in lib.mlq_last_error()
    g = mlq.make_gather(1, 0, 0, 4, [0x3000], [0x4000], epoch=1)
    g.defer_wait = 2
    op = mlq.linear_op("q8_0", 0x1000, 4, 32, 0x2000, 1, 0x3000, gather=g)
    arr = (mlq.LinearOp * 1)(op)
    assert lib.mlq_linear_batch(arr, 1, None) == 10
    assert b"defer_wait" in lib.mlq_last_error()


def test_joins_run_follows_the_header_rule(pkg):
    """mlq.joins_run (the bench's mirror of which batch ops join a run
    launch) follows include/mlq.h's rule: one row of x, in_features % 4 == 0,
    a row pitch that is a multiple of 16 bytes, and (q8_0, q4_0) an even
    block count per row."""
    mlq = pkg.mlq
    for fmt, bb in (("q8_0", 34), ("q4_0", 18), ("q4_1", 20)):
        for in_f in (128, 896, 1024, 1152, 1280, 2048, 2112, 3584, 4096, 4100, 14336, 18944):
            bpr = (in_f + 31) // 32
            want = in_f % 4 == 0 and (bpr * bb) % 16 == 0 and (fmt == "q4_1" or bpr % 2 == 0)
            assert mlq.joins_run(fmt, 1, in_f) == want, (fmt, in_f)
            assert not mlq.joins_run(fmt, 2, in_f)
    # the bench's decode step: every product joins
    assert all(mlq.joins_run("q4_0", 1, i) for i in (3584, 18944))
