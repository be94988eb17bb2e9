"""mlq_gguf_upload_rows on the GPU: blocks from a GGUF file straight into
device memory -- byte-identical to the file (the reference reads the same
bytes, tests/test_gguf.py) -- whole and as row shards, then used as the
weights of mlq_linear and checked against the oracle (relative L2 1e-3 per
output row)."""
from __future__ import annotations

import numpy as np
import pytest

import gguf_writer as gw
from conftest import rel_l2_rows

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("fmt,gtype,out_f,in_f", [("q8_0", 8, 4864, 896), ("q4_0", 2, 3000, 3584),
                                                  ("q4_1", 3, 1000, 4096)])
def test_upload_whole_and_sharded(tmp_path, oracle, pkg, fmt, gtype, out_f, in_f):
    mlq = pkg.mlq
    blocks = gw.quantized(oracle, fmt, out_f, in_f, 7, pkg.synth)
    # a second tensor first, so the matrix sits at a non-zero offset
    raw = gw.build([], [("norm", [in_f], 0, np.ones(in_f, np.float32).tobytes()),
                        ("w", [in_f, out_f], gtype, blocks)], alignment=64)
    path = tmp_path / "w.gguf"
    path.write_bytes(raw)
    nbytes = len(blocks)
    with mlq.GgufFile(path) as g:
        i = g.find("w")
        t = g.info(i)
        assert t["rows"] == out_f and t["nbytes"] == nbytes
        whole = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        g.upload_rows(i, 0, out_f, whole.data_ptr(), nbytes)
        assert bytes(whole.cpu().numpy()) == blocks
        # three row shards (the ranks of a row-sharded model), uploaded apart
        cuts = [0, 8 * (out_f // 24), 8 * (out_f // 12), out_f]
        parts = []
        for b, e in zip(cuts[:-1], cuts[1:]):
            dst = torch.empty((e - b) * t["row_bytes"], dtype=torch.uint8, device="cuda")
            g.upload_rows(i, b, e, dst.data_ptr(), dst.numel())
            parts.append(dst)
        assert torch.equal(torch.cat(parts), whole)
    x = pkg.synth.normal((3, in_f), seed=8)
    y = mlq.linear(fmt, whole, out_f, in_f, torch.from_numpy(x).cuda()).cpu().numpy()
    ref = oracle.linear(fmt, x, np.frombuffer(blocks, np.uint8), out_f)
    assert rel_l2_rows(y, ref).max() <= 1e-3


def test_upload_larger_than_staging(tmp_path, oracle, pkg):
    """A 19 MB tensor goes through the two 8 MiB staging buffers in three
    chunks, alternating; every byte must land."""
    mlq = pkg.mlq
    out_f, in_f = 1100, 16384
    blocks = gw.quantized(oracle, "q8_0", out_f, in_f, 9, pkg.synth)
    path = tmp_path / "big.gguf"
    path.write_bytes(gw.build([], [("w", [in_f, out_f], 8, blocks)]))
    with mlq.GgufFile(path) as g:
        dst = torch.empty(len(blocks), dtype=torch.uint8, device="cuda")
        g.upload_rows(0, 0, out_f, dst.data_ptr(), dst.numel())
        assert bytes(dst.cpu().numpy()) == blocks
