"""Host logic of the row-sharded path, on CPU: shard planning and the
IPC-handle exchange of PeerGroup, run as world_size-2 gloo process groups
(the device calls are replaced by a recorder; nothing touches a GPU)."""
from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp


def test_shard_rows_cover_and_align(pkg):
    import importlib
    sh = importlib.import_module("mini_llama_b200.sharding")
    for out, world in [(152064, 8), (18944, 4), (3584, 2), (100, 3), (8, 8), (4864, 1)]:
        ranges = sh.shard_rows(out, world)
        sh.check_partition(ranges, out)
        for b, e in ranges[:-1]:
            assert b % 8 == 0 and e % 8 == 0
    r = sh.shard_rows(4608, 4, owners=[0])
    assert r[0] == (0, 4608) and all(b == e for b, e in r[1:])
    sh.check_partition(r, 4608)
    with pytest.raises(ValueError):
        sh.check_partition([(0, 10), (12, 20)], 20)
    with pytest.raises(ValueError):
        sh.check_partition([(0, 10), (8, 20)], 20)


class FakeMlq:
    """Stands in for the library's peer-memory calls (host logic only)."""

    def __init__(self, rank):
        self.rank, self.next, self.opened, self.closed, self.freed = rank, 0, [], [], []

    def peer_alloc(self, nbytes):
        self.next += 1
        ptr = (self.rank + 1) * 0x1000000 + self.next * 0x1000
        return ptr, ptr.to_bytes(8, "little") * 8

    def peer_open(self, handle):
        ptr = int.from_bytes(handle[:8], "little") + 0x100  # "mapped" address
        self.opened.append(ptr)
        return ptr

    def peer_close(self, ptr):
        self.closed.append(ptr)

    def peer_free(self, ptr):
        self.freed.append(ptr)


def _worker(rank, world, port, q):
    import importlib.util
    import sys
    from pathlib import Path

    import torch.distributed as dist
    root = Path(__file__).resolve().parents[1]
    spec = importlib.util.spec_from_file_location(
        "mini_llama_b200", root / "mini-llama_b200" / "__init__.py",
        submodule_search_locations=[str(root / "mini-llama_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mini_llama_b200"] = mod
    spec.loader.exec_module(mod)
    sh = importlib.import_module("mini_llama_b200.sharding")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fake = FakeMlq(rank)
    group = sh.PeerGroup(fake, dist, rank, world)
    buf = group.alloc(256)
    ranges = sh.shard_rows(1000, world)
    lin = sh.ShardedLinear(fake, "q4_0", 1000, 64, 1, ranges, rank, group, buf)
    result = {"local": buf.local, "peers": buf.peers, "range": (lin.begin, lin.end),
              "y0": lin.y_ptr(2), "y1": lin.y_ptr(3)}
    group.close()
    result["closed"] = len(fake.closed)
    result["freed"] = len(fake.freed)
    q.put((rank, result))
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_peer_group_exchange_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every rank sees its own buffer as-is and each peer's through a mapping
    for r in range(2):
        other = 1 - r
        assert res[r]["peers"][r] == res[r]["local"]
        assert res[r]["peers"][other] == res[other]["local"] + 0x100
        assert res[r]["closed"] == 3 and res[r]["freed"] == 3  # flags + two y buffers
    assert res[0]["range"] == (0, 496) and res[1]["range"] == (496, 1000)
    assert res[0]["y0"] != res[0]["y1"]  # consecutive epochs alternate y buffers


def _plan_worker(rank, world, port, q):
    """One gloo rank: the bench's step bookkeeping (StepPlan + GatherSlab) for
    a Qwen2-7B step with the FFN and lm_head sharded; records what each rank
    would launch (epochs, y parities, peer y pointers)."""
    import importlib.util
    import sys
    from pathlib import Path

    import torch.distributed as dist
    root = Path(__file__).resolve().parents[1]
    spec = importlib.util.spec_from_file_location(
        "mini_llama_b200", root / "mini-llama_b200" / "__init__.py",
        submodule_search_locations=[str(root / "mini-llama_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mini_llama_b200"] = mod
    spec.loader.exec_module(mod)
    sh = importlib.import_module("mini_llama_b200.sharding")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fake = FakeMlq(rank)
    group = sh.PeerGroup(fake, dist, rank, world)
    mats = [("qkv", 4608, 3584), ("o", 3584, 3584), ("gate", 18944, 3584), ("up", 18944, 3584),
            ("down", 3584, 18944), ("lm_head", 152064, 3584)]
    plan = sh.StepPlan(mats, world, rank, shard={"gate", "up", "down", "lm_head"})
    slab = sh.GatherSlab(group, [4 * o for n, o, _ in mats if plan.place[n] == "shard"])
    steps = [plan.next_step() for _ in range(3)]
    # per-op calls (the bench's per-launch timing) keep the parities in step
    singles = [plan.next_call(n) for n in plan.sharded]
    after = plan.next_step()
    res = {"active": [n for n, _, _ in mats if plan.active(n)], "rows": {n: plan.rows(n) for n, _, _ in mats},
           "steps": steps, "singles": singles, "after": after,
           "y": [[slab.peer_ptrs(p, k) for k in range(len(plan.sharded))] for p in (0, 1)],
           "local": [slab.local_ptr(p, 0) for p in (0, 1)]}
    # a later plan on the same flag words continues the epoch sequence
    nxt = sh.StepPlan(mats, world, rank, shard={"gate", "lm_head"}, epoch0=plan.epoch)
    res["next_plan"] = (plan.epoch, nxt.next_step())
    plan.calls["gate"] += 1  # unequal call counts cannot form a step
    try:
        plan.next_step()
        res["unequal_raised"] = False
    except RuntimeError:
        res["unequal_raised"] = True
    group.close()
    q.put((rank, res))
    dist.destroy_process_group()


def test_step_plan_gloo():
    """Both ranks agree on the epoch sequence and y parities of every sharded
    call, rank 0 alone runs the small matrices, and each sharded matrix's y
    slices sit in the two IPC allocations at the same offsets on every rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_plan_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    r0, r1 = res[0], res[1]
    assert r0["active"] == ["qkv", "o", "gate", "up", "down", "lm_head"]
    assert r1["active"] == ["gate", "up", "down", "lm_head"]
    assert r0["rows"]["qkv"] == (0, 4608) and r1["rows"]["qkv"] == (4608, 4608)
    assert r0["rows"]["lm_head"] == (0, 76032) and r1["rows"]["lm_head"] == (76032, 152064)
    # three steps of four sharded calls: epochs 1..12, parities 0, 1, 0
    assert r0["steps"] == r1["steps"]
    assert [p for p, _ in r0["steps"]] == [0, 1, 0]
    last, (par, eps) = r0["next_plan"]
    assert r0["next_plan"] == r1["next_plan"] and par == 0 and eps == [last + 1, last + 2]
    assert [e for _, es in r0["steps"] for e in es] == list(range(1, 13))
    assert r0["singles"] == r1["singles"] == [(13, 1), (14, 1), (15, 1), (16, 1)]
    assert r0["after"] == r1["after"] == (0, [17, 18, 19, 20])
    for r in (0, 1):
        ys = res[r]["y"]
        assert len(ys[0]) == 4 and ys[0][0] != ys[1][0]     # the parities' buffers differ
        assert ys[0][1][0] - ys[0][0][0] == 4 * 18944        # gate's slice, then up's
        assert ys[0][0][r] == res[r]["local"][0]             # own entry = local buffer
        assert res[r]["unequal_raised"]
    # rank 0's mapping of rank 1's buffer = rank 1's buffer (the fake maps at +0x100)
    assert r0["y"][0][2][1] == r1["y"][0][2][1] + 0x100
