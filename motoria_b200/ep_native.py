"""The expert-parallel MoE block of libmiag (miag_ep_*): NCCL and the whole
sharded step inside the library, so a C engine runs it with no other
runtime.  This module is its ctypes mirror for the tests and the bench;
rank 0 creates the NCCL id and the caller shares it with the other ranks
by any means (here a torch.distributed object broadcast, plumbing only).

The reference runs moe() (src/model/forward.c:167-197) on one device; the
outputs of the sharded block equal the one-GPU block bit for bit.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    err = N.errbuf()
    N.check(N.lib().miag_nccl_unique_id(buf, err, len(err)), err, "miag_nccl_unique_id")
    return bytes(buf.raw)


class NcclComm:
    """This rank's NCCL communicator, created by libmiag (ncclCommInitRank)."""

    def __init__(self, uid: bytes, n_ranks: int, rank: int, device: int):
        self.handle = C.c_void_p()
        idb = C.create_string_buffer(uid, 128)
        err = N.errbuf()
        N.check(N.lib().miag_nccl_comm_init(C.byref(self.handle), n_ranks, idb, rank, device,
                                            err, len(err)), err, "miag_nccl_comm_init")

    def close(self) -> None:
        if self.handle:
            N.lib().miag_nccl_comm_destroy(self.handle)
            self.handle = C.c_void_p()


class ExpertParallelBlock:
    """miag_ep over one MoEEngine: forward() is the sharded moe() step."""

    def __init__(self, engine, comm: NcclComm, placement: str = "contiguous"):
        if placement not in ("contiguous", "strided"):
            raise ValueError(f"unknown placement {placement!r}")
        self.eng, self.comm = engine, comm
        self.placement = placement
        self._ep = C.c_void_p()
        err = N.errbuf()
        N.check(N.lib().miag_ep_open(C.byref(self._ep), engine.handle, comm.handle,
                                     int(placement == "strided"), err, len(err)), err,
                "miag_ep_open")
        r, n, first, count, step = (C.c_int() for _ in range(5))
        N.lib().miag_ep_rank(self._ep, C.byref(r), C.byref(n), C.byref(first), C.byref(count),
                             C.byref(step))
        self.rank, self.world = r.value, n.value
        self._experts = list(range(first.value, first.value + count.value * step.value,
                                   step.value))

    def experts(self) -> list[int]:
        """The experts this rank's store must hold."""
        return list(self._experts)

    def forward_device(self, x_ptr: int, n_tokens: int, layer: int = 0,
                       stream: int | None = None) -> None:
        err = N.errbuf()
        N.check(N.lib().miag_moe_ep_async(self._ep, layer, C.c_void_p(x_ptr), n_tokens,
                                          C.c_void_p(stream or 0), err, len(err)), err,
                "miag_moe_ep_async")

    def forward_host(self, x: np.ndarray, layer: int = 0) -> None:
        """x [T][dim] f32 on the host, updated in place."""
        if x.dtype != np.float32 or not x.flags["C_CONTIGUOUS"] or x.ndim != 2:
            raise ValueError("x must be a C-contiguous float32 [T][dim] array")
        err = N.errbuf()
        N.check(N.lib().miag_moe_ep(self._ep, layer, x.ctypes.data, x.shape[0], err, len(err)),
                err, "miag_moe_ep")

    def last_received(self) -> tuple[int, int]:
        rows, pairs = C.c_int(), C.c_int()
        N.lib().miag_ep_last_received(self._ep, C.byref(rows), C.byref(pairs))
        return rows.value, pairs.value

    def close(self) -> None:
        if self._ep:
            N.lib().miag_ep_close(self._ep)
            self._ep = C.c_void_p()
