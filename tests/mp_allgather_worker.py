"""One rank of the multi-GPU allgather test (launched by
tests/test_allgather_gpu.py through torchrun, one process per GPU).

Every rank holds its row shard of each matrix (drawn on its GPU from the
matrix's seed at the shard's offset and quantized there), calls the fused
shard-GEMV + gather three times (the third as a batch op with a deferred
wait, then mlq_gather_wait), and checks the FULL y on its own GPU
against the CPU oracle: every row for matrices up to 8192 rows, otherwise a
sample of rows that includes every shard's first and last row.  The cases
include the BASELINE config-5 shapes (Llama-3-70B lm_head 128256x8192 and
gate 28672x8192, q4_0, batch 1 and 8).  A last phase runs three sharded
matrices and a local one as one batch (one persistent run launch per rank)."""
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

CASES = [("q4_0", 4096, 3584, 1, None), ("q8_0", 1000, 4096, 3, None),
         ("q4_1", 2048, 1024, 8, None), ("q4_0", 4608, 3584, 1, [0]),
         ("q8_0", 1536, 2048, 16, None),
         ("q4_0", 128256, 8192, 1, None), ("q4_0", 128256, 8192, 8, None),
         ("q4_0", 28672, 8192, 1, None), ("q4_0", 28672, 8192, 8, None)]


def sample_rows(out_f, ranges):
    if out_f <= 8192:
        return np.arange(out_f)
    rows = set(np.linspace(0, out_f - 1, 384).astype(int).tolist())
    for b, e in ranges:
        if e > b:
            rows.update((b, e - 1))
    return np.array(sorted(rows))


def run_phase(mlq, orc, group, flags, rank, world, dev, stream, epoch):
    """A batch the library runs as one persistent launch: four row-sharded
    one-row q4_0 matrices (deferred gathers sharing the flag words; the last
    one's rows all on rank 0, so every other rank's op has an empty shard)
    and one local matrix, then one mlq_gather_wait for the highest epoch
    (the middle step instead waits inside the run launch); three steps,
    every full y checked on this rank against the oracle."""
    fmt = "q4_0"
    mats = [(4608, 3584, None), (18944, 3584, None), (3584, 18944, None), (1024, 3584, [0])]
    lins, shards, blocks, checks = [], [], [], []
    for k, (out_f, in_f, owners) in enumerate(mats):
        seed = 300 + k
        ranges = sh.shard_rows(out_f, world, owners=owners)
        b, e = ranges[rank]
        shard = None
        if e > b:
            w32 = pkg.synth.normal_torch((e - b, in_f), seed=seed, std=0.02, device=dev, offset=b * in_f)
            shard = mlq.quantize(fmt, w32)
            del w32
        shards.append(shard)
        check = sample_rows(out_f, [rg for rg in ranges if rg[1] > rg[0]])
        wrows = np.concatenate([pkg.synth.normal_torch((1, in_f), seed=seed, std=0.02,
                                                       offset=int(r) * in_f).numpy() for r in check])
        blocks.append(orc.quantize(fmt, wrows))
        checks.append(check)
        lins.append(sh.ShardedLinear(mlq, fmt, out_f, in_f, 1, ranges, rank, group, flags))
    lblocks = orc.quantize(fmt, pkg.synth.normal((1024, 3584), seed=310, std=0.02))
    lw = torch.from_numpy(lblocks).to(dev)
    ly = torch.empty((1, 1024), device=dev)
    worst = 0.0
    for it in range(3):
        xs = [pkg.synth.normal((1, in_f), seed=5000 + 10 * it + k) for k, (_, in_f, _) in enumerate(mats)]
        xl = pkg.synth.normal((1, 3584), seed=5100 + it)
        xds = [torch.from_numpy(x).to(dev) for x in xs]
        xld = torch.from_numpy(xl).to(dev)
        ops, gs, yptrs = [], [], []
        for k, lin in enumerate(lins):
            epoch += 1
            yb = lin.ybuf[epoch & 1]
            # steps 0 and 2: publish in the launch, wait in mlq_gather_wait;
            # step 1: the run launch itself waits for every rank
            g = mlq.make_gather(world, rank, lin.begin, lin.end, yb.peers, flags.peers, epoch=epoch,
                                defer_wait=(it != 1))
            gs.append(g)
            yptrs.append(yb.local)
            wp = shards[k].data_ptr() if shards[k] is not None else 0
            ops.append(mlq.linear_op(fmt, wp, lin.out, lin.inp, xds[k].data_ptr(), 1, yb.local, gather=g))
        ops.append(mlq.linear_op(fmt, lw.data_ptr(), 1024, 3584, xld.data_ptr(), 1, ly.data_ptr()))
        mlq.Batch(ops).run(stream)
        if it != 1:
            mlq.gather_wait(gs[-1], stream)
        torch.cuda.synchronize()
        for k, (out_f, in_f, _) in enumerate(mats):
            y = sh.device_view(yptrs[k], (1, out_f)).cpu().numpy()[:, checks[k]]
            ref = orc.linear(fmt, xs[k], blocks[k], len(checks[k]))
            err = (np.linalg.norm(y - ref, axis=1) / np.linalg.norm(ref, axis=1)).max()
            worst = max(worst, err)
            assert err <= 1e-3, (rank, "run", k, it, err)
        ref = orc.linear(fmt, xl, lblocks, 1024)
        err = (np.linalg.norm(ly.cpu().numpy() - ref, axis=1) / np.linalg.norm(ref, axis=1)).max()
        worst = max(worst, err)
        assert err <= 1e-3, (rank, "run local", it, err)
        dist.barrier()
    return epoch, worst


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    mlq = pkg.mlq
    orc = Oracle()
    group = sh.PeerGroup(mlq, dist, rank, world)
    flags = group.alloc(mlq.flag_bytes())
    stream = torch.cuda.current_stream().cuda_stream
    epoch = 0
    worst = 0.0
    for ci, (fmt, out_f, in_f, rows, owners) in enumerate(CASES):
        seed = 100 + ci
        ranges = sh.shard_rows(out_f, world, owners=owners)
        b, e = ranges[rank]
        shard = None
        if e > b:
            w32 = pkg.synth.normal_torch((e - b, in_f), seed=seed, std=0.02, device=dev, offset=b * in_f)
            shard = mlq.quantize(fmt, w32)
            del w32
        # the oracle's blocks of the checked rows (CPU draw of the same numbers)
        check = sample_rows(out_f, [rg for rg in ranges if rg[1] > rg[0]])
        wrows = np.concatenate([pkg.synth.normal_torch((1, in_f), seed=seed, std=0.02,
                                                       offset=int(r) * in_f).numpy() for r in check])
        blocks = orc.quantize(fmt, wrows)
        lin = sh.ShardedLinear(mlq, fmt, out_f, in_f, rows, ranges, rank, group, flags)
        for it in range(3):
            x = pkg.synth.normal((rows, in_f), seed=1000 * ci + it)
            xd = torch.from_numpy(x).to(dev)
            epoch += 1
            # the third call: publish in the op, wait in mlq_gather_wait
            call = lin.deferred if it == 2 else lin
            yptr = call(shard.data_ptr() if shard is not None else 0, xd.data_ptr(), epoch, stream)
            torch.cuda.synchronize()
            y = sh.device_view(yptr, (rows, out_f)).cpu().numpy()[:, check]
            ref = orc.linear(fmt, x, blocks, len(check))
            err = (np.linalg.norm(y - ref, axis=1) / np.linalg.norm(ref, axis=1)).max()
            worst = max(worst, err)
            assert err <= 1e-3, (rank, fmt, out_f, in_f, rows, it, err)
        del shard
        torch.cuda.empty_cache()
        dist.barrier()
    epoch, w_run = run_phase(mlq, orc, group, flags, rank, world, dev, stream, epoch)
    worst = max(worst, w_run)
    code = mlq.device_error(local)
    assert code == 0, code
    dist.barrier()
    group.close()
    print(f"rank {rank}: ALLGATHER OK (world {world}, worst rel-L2 {worst:.2e}, {epoch} calls)", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
