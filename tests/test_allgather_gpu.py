"""mlq_linear_allgather on one GPU: the degenerate world of one rank, and
the bounded peer wait (a second rank that never runs, so its flag is never
set: the kernel must give up after 2 s, record error code 4 and return).
The real multi-GPU run is tests/mp_allgather_worker.py, launched here with
torchrun when two or more GPUs are visible."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_l2_rows

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("fmt,out_f,in_f,rows", [("q4_0", 3000, 3584, 1), ("q8_0", 777, 1024, 3),
                                                 ("q4_1", 2048, 4096, 8), ("q4_0", 512, 2048, 16)])
def test_world_of_one_matches_oracle(oracle, pkg, fmt, out_f, in_f, rows):
    mlq = pkg.mlq
    blocks = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=31, std=0.02))
    x = pkg.synth.normal((rows, in_f), seed=32)
    w_d, x_d = dev(blocks), dev(x)
    y = torch.full((rows, out_f), 7.0, dtype=torch.float32, device="cuda")
    flags = torch.zeros(mlq.flag_bytes() // 4, dtype=torch.int32, device="cuda")
    mlq.linear_allgather(fmt, w_d.data_ptr(), blocks.size // mlq.BLOCK_BYTES[fmt], out_f, in_f, 0,
                         out_f, x_d.data_ptr(), rows, [y.data_ptr()], [flags.data_ptr()], 0, 1,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rel_l2_rows(y.cpu().numpy(), oracle.linear(fmt, x, blocks, out_f)).max() <= 1e-3
    assert mlq.device_error(0) == 0


def test_arguments_validated(pkg):
    mlq = pkg.mlq
    with pytest.raises(mlq.MLQError) as e:  # rank outside the world
        mlq.linear_allgather("q4_0", 0x1000, 4, 4, 32, 0, 4, 0x2000, 1, [0x3000], [0x4000], 1, 1, None)
    assert e.value.status == 10
    with pytest.raises(mlq.MLQError) as e:  # epoch 0
        mlq.linear_allgather("q4_0", 0x1000, 4, 4, 32, 0, 4, 0x2000, 1, [0x3000], [0x4000], 0, 0, None)
    assert e.value.status == 10
    with pytest.raises(mlq.MLQError) as e:  # shard block count
        mlq.linear_allgather("q4_0", 0x1000, 3, 4, 32, 0, 4, 0x2000, 1, [0x3000], [0x4000], 0, 1, None)
    assert e.value.status == 5
    with pytest.raises(mlq.MLQError) as e:  # null peer
        mlq.linear_allgather("q4_0", 0x1000, 4, 4, 32, 0, 4, 0x2000, 1, [0x3000, 0], [0x4000, 0x5000],
                             0, 1, None)
    assert e.value.status == 2


@pytest.mark.parametrize("rows", [1, 8])
def test_peer_that_never_signals_times_out(oracle, pkg, rows):
    """Rank 0 of a world of two whose rank 1 never runs: the handshake wait
    must end after its 2 s bound with device error code 4, and rank 0's own
    rows must still be in y.  (The flag nothing sets is the only failure
    injected; no fault, no hang.)  One row takes the streaming GEMV, eight
    the batched-decode GEMM; both end with the same handshake."""
    mlq = pkg.mlq
    fmt, out_f, in_f = "q4_0", 1024, 2048
    blocks = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=41, std=0.02))
    x = pkg.synth.normal((rows, in_f), seed=42)
    half = 512
    bpr = in_f // 32
    assert mlq.takes_bgemm(rows, half, in_f) == (rows == 8)
    w_d, x_d = dev(blocks[: half * bpr * 18]), dev(x)
    y0 = torch.zeros((rows, out_f), dtype=torch.float32, device="cuda")
    y1 = torch.zeros((rows, out_f), dtype=torch.float32, device="cuda")  # the absent peer's y
    f0 = torch.zeros(mlq.flag_bytes() // 4, dtype=torch.int32, device="cuda")
    f1 = torch.zeros(mlq.flag_bytes() // 4, dtype=torch.int32, device="cuda")
    assert mlq.device_error(0) == 0
    mlq.linear_allgather(fmt, w_d.data_ptr(), half * bpr, out_f, in_f, 0, half, x_d.data_ptr(), rows,
                         [y0.data_ptr(), y1.data_ptr()], [f0.data_ptr(), f1.data_ptr()], 0, 1,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert mlq.device_error(0) == 4
    assert mlq.device_error(0) == 0  # reading clears it
    ref = oracle.linear(fmt, x, blocks, out_f)
    assert rel_l2_rows(y0.cpu().numpy()[:, :half], ref[:, :half]).max() <= 1e-3
    assert rel_l2_rows(y1.cpu().numpy()[:, :half], ref[:, :half]).max() <= 1e-3  # stores reached the "peer"
    assert int(f1[0].item()) == 1 and int(f0[0].item()) == 1  # epoch published to both ranks


@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_allgather(world):
    """torchrun worlds of 2, 4 and 8 GPUs (each as far as the box has GPUs):
    every rank checks the gathered y against the oracle."""
    n = torch.cuda.device_count()
    if n < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(29533 + world), str(ROOT / "tests" / "mp_allgather_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=str(ROOT))
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
    assert r.stdout.count("ALLGATHER OK") == world


@pytest.mark.parametrize("rows", [1, 8])
def test_world_of_one_deferred_wait(oracle, pkg, rows):
    """A batch op with defer_wait in a world of one: mlq_gather_wait has no
    peer to wait for (stream order covers this rank) and y is complete
    after it.  One row takes the streaming GEMV, eight the batched-decode
    GEMM."""
    mlq = pkg.mlq
    fmt, out_f, in_f = "q4_0", 1000, 2048
    blocks = oracle.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=51, std=0.02))
    x = pkg.synth.normal((rows, in_f), seed=52)
    w_d, x_d = dev(blocks), dev(x)
    y = torch.full((rows, out_f), 7.0, dtype=torch.float32, device="cuda")
    flags = torch.zeros(mlq.flag_bytes() // 4, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for epoch in (1, 2, 3):
        g = mlq.make_gather(1, 0, 0, out_f, [y.data_ptr()], [flags.data_ptr()], epoch=epoch, defer_wait=True)
        op = mlq.linear_op(fmt, w_d.data_ptr(), out_f, in_f, x_d.data_ptr(), rows, y.data_ptr(), gather=g)
        mlq.Batch([op]).run(s)
        mlq.gather_wait(g, s)
        torch.cuda.synchronize()
    assert rel_l2_rows(y.cpu().numpy(), oracle.linear(fmt, x, blocks, out_f)).max() <= 1e-3
    assert mlq.device_error(0) == 0
