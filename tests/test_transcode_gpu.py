"""Model-level quantization on the device (mlq_transcode /
mlq_quantize_model, include/mlq.h): every source format to every target,
byte-identical to the reference's rule -- dequantize to fp32 with
dequantizeFrom*, then quantizeToQ80 / quantizeToQ40 (src/model.cc:94-149)
-- as the oracle (pinned to the reference's own build) computes it, on
matrices with partial last blocks and all-zero blocks."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


FMTS = ["q8_0", "q4_0", "q4_1"]


@pytest.mark.parametrize("src", FMTS)
@pytest.mark.parametrize("dst", FMTS)
@pytest.mark.parametrize("shape", [(64, 4096), (37, 100), (5, 31)])
def test_transcode_bit_exact(oracle, pkg, src, dst, shape):
    rows, cols = shape
    w = pkg.synth.normal((rows, cols), seed=rows + cols, std=0.02)
    w[1, :] = 0.0  # zero blocks
    w[2, :32] *= 1e4  # a block with a wide range
    sblocks = oracle.quantize(src, w)
    got = pkg.mlq.transcode(src, torch.from_numpy(sblocks).cuda(), dst, rows, cols).cpu().numpy()
    want = sblocks if src == dst else oracle.quantize(dst, oracle.dequantize(src, sblocks, rows, cols))
    np.testing.assert_array_equal(got, want)


def test_quantize_model_batch(oracle, pkg):
    """A model's linear weights in one call: fp32 and block sources mixed."""
    mlq = pkg.mlq
    shapes = [(128, 1024, "f32"), (64, 2048, "q4_1"), (32, 4096, "q8_0")]
    srcs, outs, wants, ops = [], [], [], []
    for i, (r, c, st) in enumerate(shapes):
        w = pkg.synth.normal((r, c), seed=90 + i, std=0.02)
        if st == "f32":
            s = torch.from_numpy(w).cuda()
            want = oracle.quantize("q4_0", w)
        else:
            b = oracle.quantize(st, w)
            s = torch.from_numpy(b).cuda()
            want = oracle.quantize("q4_0", oracle.dequantize(st, b, r, c))
        o = torch.empty(mlq.weight_bytes("q4_0", r, c), dtype=torch.uint8, device="cuda")
        srcs.append(s)
        outs.append(o)
        wants.append(want)
        ops.append(mlq.QuantizeOp(0 if st == "f32" else mlq.FORMATS[st], s.data_ptr(), mlq.FORMATS["q4_0"],
                                  o.data_ptr(), r, c))
    mlq.quantize_model(ops)
    torch.cuda.synchronize()
    for o, want in zip(outs, wants):
        np.testing.assert_array_equal(o.cpu().numpy(), want)
