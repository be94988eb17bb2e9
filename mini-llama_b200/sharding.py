"""Row sharding of quantized matrices across the GPUs of one node.

The reference keeps every weight on one device (cuda_weight_upload.h:46).
Here a large matrix's output rows are split into contiguous ranges, one per
rank; each rank keeps its range's blocks resident (a row range of the AoS
block array is a contiguous byte slice, so nothing is repacked), and
mlq_linear_allgather writes every range into every rank's y over NVLink.

Host-side pieces:
  * shard_rows(): the row ranges (multiples of 8 rows, so every shard of a
    16-byte aligned array stays 16-byte aligned);
  * PeerGroup: per-rank IPC buffers exchanged through torch.distributed
    (plain CUDA IPC mappings, no multicast objects) -- y buffers (two, used
    alternately by consecutive calls) and the 256-byte flag buffer;
  * ShardedLinear: one matrix's shard plus its call state (epoch counter);
  * StepPlan: placement of a decode step's matrices (sharded / rank 0) and
    the epoch and y-buffer bookkeeping of their calls, for batches
    (mlq_linear_batch) that launch a whole step at once;
  * GatherSlab: the sharded matrices' y buffers of a step in two IPC
    allocations (one per y parity).
"""
from __future__ import annotations

from dataclasses import dataclass


def shard_rows(out_features: int, world: int, align: int = 8, owners=None):
    """[(row_begin, row_end)] per rank, contiguous and covering [0, out).

    Rows are split as evenly as possible in units of `align` rows (the last
    rank takes the remainder).  `owners` restricts the rows to those ranks
    (e.g. [0] keeps a small matrix on rank 0; the others get empty ranges).
    """
    if out_features <= 0 or world <= 0:
        raise ValueError("out_features and world must be positive")
    owners = list(range(world)) if owners is None else list(owners)
    if not owners or any(r < 0 or r >= world for r in owners):
        raise ValueError("owners must be ranks of the world")
    units = (out_features + align - 1) // align
    n = len(owners)
    bounds = [min(out_features, (units * i // n) * align) for i in range(n + 1)]
    bounds[-1] = out_features
    ranges = [(0, 0)] * world
    for i, r in enumerate(owners):
        ranges[r] = (bounds[i], bounds[i + 1])
    # ranks that own nothing get an empty range at the end of the matrix
    return [rg if r in owners else (out_features, out_features) for r, rg in enumerate(ranges)]


def check_partition(ranges, out_features: int) -> None:
    """Raises unless the non-empty ranges tile [0, out_features) exactly."""
    spans = sorted((b, e) for b, e in ranges if e > b)
    pos = 0
    for b, e in spans:
        if b != pos:
            raise ValueError(f"row ranges leave a gap or overlap at row {pos}")
        pos = e
    if pos != out_features:
        raise ValueError(f"row ranges end at {pos}, not {out_features}")


@dataclass
class PeerBuffer:
    local: int          # this rank's allocation (device pointer)
    peers: list         # every rank's buffer mapped here (peers[rank] == local)


class PeerGroup:
    """IPC-shared buffers of one process group (one process per GPU)."""

    def __init__(self, mlq, dist, rank: int, world: int):
        self.mlq, self.dist, self.rank, self.world = mlq, dist, rank, world
        self.opened, self.owned = [], []

    def alloc(self, nbytes: int) -> PeerBuffer:
        ptr, handle = self.mlq.peer_alloc(nbytes)
        self.owned.append(ptr)
        handles = [None] * self.world
        self.dist.all_gather_object(handles, handle)
        peers = []
        for r, h in enumerate(handles):
            if r == self.rank:
                peers.append(ptr)
            else:
                p = self.mlq.peer_open(h)
                self.opened.append(p)
                peers.append(p)
        return PeerBuffer(ptr, peers)

    def close(self) -> None:
        for p in self.opened:
            self.mlq.peer_close(p)
        self.opened = []
        self.dist.barrier()  # no peer still maps our memory past this point
        for p in self.owned:
            self.mlq.peer_free(p)
        self.owned = []


class ShardedLinear:
    """One row-sharded matrix on this rank and its all-gather call."""

    def __init__(self, mlq, fmt: str, out_features: int, in_features: int, rows: int,
                 ranges, rank: int, group: PeerGroup, flags: PeerBuffer):
        check_partition(ranges, out_features)
        self.mlq, self.fmt = mlq, fmt
        self.out, self.inp, self.rows = out_features, in_features, rows
        self.rank, self.world = rank, len(ranges)
        self.begin, self.end = ranges[rank]
        self.bpr = (in_features + 31) // 32
        self.shard_blocks = (self.end - self.begin) * self.bpr
        self.flags = flags
        ybytes = 4 * rows * out_features
        self.ybuf = [group.alloc(ybytes), group.alloc(ybytes)]  # alternate per call

    def y_ptr(self, epoch: int) -> int:
        return self.ybuf[epoch & 1].local

    def __call__(self, w_shard_ptr: int, x_ptr: int, epoch: int, stream: int | None) -> int:
        """Launches the fused shard GEMV + gather; returns the local y pointer."""
        yb = self.ybuf[epoch & 1]
        self.mlq.linear_allgather(self.fmt, w_shard_ptr, self.shard_blocks, self.out, self.inp,
                                  self.begin, self.end, x_ptr, self.rows, yb.peers,
                                  self.flags.peers, self.rank, epoch, stream)
        return yb.local

    def deferred(self, w_shard_ptr: int, x_ptr: int, epoch: int, stream: int | None) -> int:
        """The same product as a batch op that only publishes its epoch,
        then the separate wait (mlq_gather_wait); returns the local y."""
        yb = self.ybuf[epoch & 1]
        g = self.mlq.make_gather(self.world, self.rank, self.begin, self.end, yb.peers, self.flags.peers,
                                 epoch=epoch, defer_wait=True)
        op = self.mlq.linear_op(self.fmt, w_shard_ptr, self.out, self.inp, x_ptr, self.rows, yb.local, gather=g)
        self.mlq.Batch([op]).run(stream)
        self.mlq.gather_wait(g, stream)
        return yb.local


class _CudaArray:
    __slots__ = ("__cuda_array_interface__",)

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape),
                                         "typestr": typestr, "version": 3, "strides": None}


def device_view(ptr: int, shape, dtype="float32"):
    """A torch CUDA tensor viewing `ptr` (no copy; the memory stays owned by
    whoever allocated it)."""
    import torch
    typestr = {"float32": "<f4", "int32": "<i4", "uint8": "|u1"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device="cuda")


class StepPlan:
    """Placement and call bookkeeping of one decode step's matrices.

    matrices: [(name, out_features, in_features)] in call order.  At world 1
    every matrix runs locally.  At world > 1 a matrix named in `shard` is
    row-sharded across every rank (fused gather); any other runs on rank 0
    alone ("local0"), as north_star places small matrices on one GPU.

    Sharded calls share one flag buffer per rank, so their epochs form one
    sequence: every sharded call takes the next epoch, in the same order on
    every rank.  Each sharded matrix alternates between two y buffers
    (parity = how many times it was called, mod 2), so a rank that runs
    ahead never writes a y that a slower peer may still be reading.
    """

    def __init__(self, matrices, world: int, rank: int, shard=(), epoch0: int = 0):
        """epoch0: the last epoch already published on the flag words these
        calls use (a plan that follows another on the same flags continues
        its sequence; a restarted sequence would find its waits satisfied by
        the older, higher epochs)."""
        self.matrices = list(matrices)
        self.world, self.rank = world, rank
        self.place, self.ranges = {}, {}
        for name, out_f, _ in self.matrices:
            if world == 1:
                self.place[name] = "local"
                self.ranges[name] = [(0, out_f)]
            elif name in shard:
                self.place[name] = "shard"
                self.ranges[name] = shard_rows(out_f, world)
            else:
                self.place[name] = "local0"
                self.ranges[name] = shard_rows(out_f, world, owners=[0])
        self.sharded = [n for n, _, _ in self.matrices if self.place[n] == "shard"]
        self.epoch = epoch0
        self.calls = {n: 0 for n in self.sharded}

    def rows(self, name):
        """This rank's (row_begin, row_end) of the matrix."""
        rg = self.ranges[name]
        return rg[self.rank] if self.world > 1 else rg[0]

    def active(self, name) -> bool:
        """Whether this rank makes a call for the matrix (sharded: every rank,
        also one that owns no rows; local0: rank 0 only)."""
        return self.place[name] in ("local", "shard") or self.rank == 0

    def next_call(self, name):
        """(epoch, y parity) of the matrix's next sharded call."""
        self.epoch += 1
        parity = self.calls[name] & 1
        self.calls[name] += 1
        return self.epoch, parity

    def next_step(self):
        """(y parity, [epoch per sharded matrix in call order]) of a whole step;
        every sharded matrix must have been called equally often so far."""
        counts = {self.calls[n] for n in self.sharded}
        if len(counts) > 1:
            raise RuntimeError("sharded matrices were called unequally often; a step needs one parity")
        out = [self.next_call(n) for n in self.sharded]
        return (out[0][1] if out else 0), [e for e, _ in out]


class GatherSlab:
    """The y buffers of every sharded matrix of a step, for both parities: two
    IPC allocations (one per parity) sliced per matrix, 256-B aligned."""

    def __init__(self, group: PeerGroup, nbytes_per_matrix):
        self.offsets, off = [], 0
        for nb in nbytes_per_matrix:
            self.offsets.append(off)
            off += (nb + 255) // 256 * 256
        self.total = max(off, 256)
        self.bufs = [group.alloc(self.total), group.alloc(self.total)]

    def peer_ptrs(self, parity: int, k: int):
        """Every rank's y of matrix k (parity buffer), mapped here."""
        return [p + self.offsets[k] for p in self.bufs[parity].peers]

    def local_ptr(self, parity: int, k: int) -> int:
        return self.bufs[parity].local + self.offsets[k]
