"""One rank of the multi-GPU allgather test (launched by
tests/test_allgather_gpu.py through torchrun, one process per GPU).

Every rank holds its row shard of each matrix, calls the fused shard-GEMV +
gather, and checks the FULL y on its own GPU against the CPU oracle."""
from __future__ import annotations

import importlib
import importlib.util
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
spec = importlib.util.spec_from_file_location(
    "mini_llama_b200", ROOT / "mini-llama_b200" / "__init__.py",
    submodule_search_locations=[str(ROOT / "mini-llama_b200")])
pkg = importlib.util.module_from_spec(spec)
sys.modules["mini_llama_b200"] = pkg
spec.loader.exec_module(pkg)
sh = importlib.import_module("mini_llama_b200.sharding")
from oracle.oracle import Oracle  # noqa: E402  (the checker)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    mlq = pkg.mlq
    orc = Oracle()
    group = sh.PeerGroup(mlq, dist, rank, world)
    flags = group.alloc(mlq.flag_bytes())
    stream = torch.cuda.current_stream().cuda_stream
    epoch = 0
    cases = [("q4_0", 4096, 3584, 1, None), ("q8_0", 1000, 4096, 3, None),
             ("q4_1", 2048, 1024, 8, None), ("q4_0", 4608, 3584, 1, [0]),
             ("q8_0", 1536, 2048, 16, None)]
    worst = 0.0
    for ci, (fmt, out_f, in_f, rows, owners) in enumerate(cases):
        blocks = orc.quantize(fmt, pkg.synth.normal((out_f, in_f), seed=100 + ci, std=0.02))
        ranges = sh.shard_rows(out_f, world, owners=owners)
        b, e = ranges[rank]
        rb = (in_f // 32) * mlq.BLOCK_BYTES[fmt]
        shard = torch.from_numpy(blocks[b * rb:e * rb].copy()).to(dev) if e > b else None
        lin = sh.ShardedLinear(mlq, fmt, out_f, in_f, rows, ranges, rank, group, flags)
        for it in range(3):
            x = pkg.synth.normal((rows, in_f), seed=1000 * ci + it)
            xd = torch.from_numpy(x).to(dev)
            epoch += 1
            yptr = lin(shard.data_ptr() if shard is not None else 0, xd.data_ptr(), epoch, stream)
            torch.cuda.synchronize()
            y = sh.device_view(yptr, (rows, out_f)).cpu().numpy()
            ref = orc.linear(fmt, x, blocks, out_f)
            err = (np.linalg.norm(y - ref, axis=1) / np.linalg.norm(ref, axis=1)).max()
            worst = max(worst, err)
            assert err <= 1e-3, (rank, fmt, out_f, in_f, rows, it, err)
        dist.barrier()
    code = mlq.device_error(local)
    assert code == 0, code
    dist.barrier()
    group.close()
    print(f"rank {rank}: ALLGATHER OK (worst rel-L2 {worst:.2e}, {epoch} calls)", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
