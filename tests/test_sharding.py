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
