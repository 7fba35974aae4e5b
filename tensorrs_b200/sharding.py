"""Host side of the several-GPU path: one process per GPU, each holding a
leading-dimension (dim-0) shard of every tensor.

* `shard_rows` splits `total` rows over `world` ranks: the first
  `total % world` ranks take one row more, so every split is a contiguous run
  of global rows and ranks may hold zero rows.
* `Communicator` creates the library's NCCL communicator (trs_comm_init_rank)
  after the unique id made on rank 0 (trs_comm_unique_id) has been broadcast
  over an already initialised torch.distributed process group (any backend;
  gloo keeps NCCL out of torch).  Creation is bounded by `timeout_ms`: a rank
  that never joins makes the others fail with TRS_ERR_TIMEOUT.
* The sharded calls (trs_sharded_sum, trs_sharded_elementwise_sum,
  trs_sharded_sum_axis0, trs_sharded_max_axis0, trs_sharded_argmax_axis0)
  leave the global result on every rank.

The reference is single-process (tensorrs has no multi-device code); the
sharded calls return what sum (base.rs:1024), sum_axis(0) (base.rs:1051),
max_axis(0) (base.rs:1396) and argmax_axis(0) (base.rs:1458) return on the
unsplit tensor.
"""
from __future__ import annotations

import ctypes

from . import abi

UNIQUE_ID_BYTES = 128


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """(first global row, row count) of `rank`'s shard of `total` rows."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad split: total={total} world={world} rank={rank}")
    base, extra = divmod(total, world)
    rows = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, rows


def row_offsets(counts: list[int]) -> list[int]:
    """Global index of each rank's first row given every rank's row count
    (the argmax index base of that rank)."""
    out, acc = [], 0
    for c in counts:
        out.append(acc)
        acc += int(c)
    return out


def exchange_unique_id(make_id, rank: int, dist) -> bytes:
    """Rank 0 calls `make_id()` (128 bytes); every rank returns rank 0's id,
    broadcast through torch.distributed `dist`."""
    obj = [bytes(make_id()) if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != UNIQUE_ID_BYTES:
        raise RuntimeError("communicator id exchange returned a malformed id")
    return bytes(uid)


def library_unique_id(lib) -> bytes:
    buf = (ctypes.c_uint8 * UNIQUE_ID_BYTES)()
    abi.check(lib.trs_comm_unique_id(buf))
    return bytes(buf)


class Communicator:
    """The library's NCCL communicator for this rank (trs_comm*)."""

    def __init__(self, lib, rank: int, world: int, dist, timeout_ms: int = 120000):
        self.lib = lib
        self.rank = rank
        self.world = world
        uid = exchange_unique_id(lambda: library_unique_id(lib), rank, dist)
        arr = (ctypes.c_uint8 * UNIQUE_ID_BYTES).from_buffer_copy(uid)
        self.handle = ctypes.c_void_p()
        abi.check(lib.trs_comm_init_rank(arr, world, rank, int(timeout_ms), ctypes.byref(self.handle)))

    @property
    def peer_exchange(self) -> bool:
        """True when the sharded sums combine over NVLink peer memory."""
        v = ctypes.c_int32(0)
        abi.check(self.lib.trs_comm_peer_exchange(self.handle, ctypes.byref(v)))
        return bool(v.value)

    def destroy(self) -> None:
        if self.handle:
            abi.check(self.lib.trs_comm_destroy(self.handle))
            self.handle = ctypes.c_void_p()

    def abort(self) -> None:
        if self.handle:
            self.lib.trs_comm_abort(self.handle)
            self.handle = ctypes.c_void_p()

    # -- the sharded calls (views over this rank's shard, results global) --
    def sum(self, shard: abi.View, out: abi.View, stream: int) -> None:
        abi.check(self.lib.trs_sharded_sum(self.handle, ctypes.byref(shard), ctypes.byref(out), stream))

    def elementwise_sum(self, prog: abi.Program, ins, out: abi.View | None, sum_out: abi.View, stream: int) -> None:
        arr = abi.views_array(list(ins))
        outp = ctypes.byref(out) if out is not None else None
        abi.check(self.lib.trs_sharded_elementwise_sum(self.handle, ctypes.byref(prog), arr, outp,
                                                       ctypes.byref(sum_out), stream))

    def sum_axis0(self, shard: abi.View, out: abi.View, stream: int) -> None:
        abi.check(self.lib.trs_sharded_sum_axis0(self.handle, ctypes.byref(shard), ctypes.byref(out), stream))

    def max_axis0(self, shard: abi.View, out: abi.View, stream: int) -> None:
        abi.check(self.lib.trs_sharded_max_axis0(self.handle, ctypes.byref(shard), ctypes.byref(out), stream))

    def argmax_axis0(self, shard: abi.View, out: abi.View, stream: int) -> None:
        abi.check(self.lib.trs_sharded_argmax_axis0(self.handle, ctypes.byref(shard), ctypes.byref(out), stream))
