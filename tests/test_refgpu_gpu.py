"""This library's kernels against the REFERENCE's own CUDA kernels
(q80/q40/q41LinearKernel of src/cuda_quant.cu, built for sm_100a into
oracle/_ref/libref_gpu.so) on the same device weights and x: every output
vector within relative L2 1e-3 (the two sum in different fp32 orders), for
every format, at the BASELINE config-1/2/3 shapes, decode and batched."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2_rows

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def refgpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oracle.oracle import ReferenceGpu
    if not ReferenceGpu.available():
        pytest.skip("oracle/_ref/libref_gpu.so not built (needs the reference checkout)")
    return ReferenceGpu()


@pytest.mark.parametrize("fmt,out_f,in_f", [("q8_0", 4864, 896), ("q4_0", 4608, 3584), ("q4_0", 3584, 18944),
                                            ("q4_1", 14336, 4096), ("q8_0", 1000, 100)])
def test_against_reference_kernels(pkg, refgpu, fmt, out_f, in_f):
    mlq = pkg.mlq
    w32 = pkg.synth.normal_torch((out_f, in_f), seed=77, std=0.02, device="cuda")
    w = mlq.quantize(fmt, w32)
    for rows in (1, 3, 16):
        x = torch.from_numpy(pkg.synth.normal((rows, in_f), seed=78 + rows)).cuda()
        y_ref = torch.full((rows, out_f), float("nan"), device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        refgpu.linear(fmt, x.data_ptr(), w.data_ptr(), y_ref.data_ptr(), rows, in_f, out_f, s)
        y = mlq.linear(fmt, w, out_f, in_f, x)
        torch.cuda.synchronize()
        err = rel_l2_rows(y.cpu().numpy(), y_ref.cpu().numpy()).max()
        assert err <= 1e-3, (fmt, out_f, in_f, rows, err)
