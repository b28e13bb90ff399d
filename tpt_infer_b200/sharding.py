"""Multi-GPU plumbing: one process per GPU on one node.

Two ways of spreading the model workloads over P GPUs:

- batch sharding (MLP, ResNet-18, BERT): rank r runs the whole model on its
  contiguous slice of the batch (``batch_shard``); weights are replicated and
  uploaded once per GPU; there is no collective on the data path.
- FFN column sharding (the BERT variant): every rank holds the whole token
  batch; the FFN1 weight W1^T [3072, 768] is split along its output channels
  (the per-channel quantization axis, ``column_shard``), each rank computes
  GELU(X W1_r + b1_r) for its 3072/P channels, quantizes it with the scale of
  the whole tensor (a max over the ranks at calibration), and an NCCL
  all-gather inside the plan reassembles [P][T][3072/P] int8 panels, which a
  relayout turns into the [T][3072] rows FFN2 consumes. The result is
  bit-identical to the unsharded plan: W8A8 outputs are exact per channel and
  the scale is the same.

The communicator is the library's own (``tpt_cuda_comm_*``, NCCL); its unique
id travels from rank 0 to the others over any channel the caller has, e.g.
``torch.distributed.broadcast_object_list``.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._capi import COMM_ID_BYTES, lib
from .backend import OK, OpError


def batch_shard(total: int, world: int, rank: int):
    """(start, count) of rank's contiguous slice of ``total`` items; the first
    ``total % world`` ranks take one extra item."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def column_shard(n: int, world: int, rank: int):
    """(start, count) of rank's output channels of an n-channel weight. The
    all-gather reassembles equal panels, so n must divide evenly."""
    if n % world:
        raise ValueError(f"{n} output channels do not split evenly over {world} ranks")
    c = n // world
    return rank * c, c


def slice_qlinear(ql, start: int, count: int):
    """Rows [start, start + count) of a per-output-channel INT8 weight."""
    from .graphs import QLinear

    return QLinear(count, ql.k, np.ascontiguousarray(ql.q[start:start + count]),
                   np.ascontiguousarray(ql.scales[start:start + count]),
                   np.ascontiguousarray(ql.bias[start:start + count]))


def panels_to_rows(panels: np.ndarray, P: int, T: int, C_: int) -> np.ndarray:
    """Host statement of TPT_OP_PANELS_TO_ROWS: [P][T][C] -> [T][P*C]."""
    return np.ascontiguousarray(panels.reshape(P, T, C_).transpose(1, 0, 2).reshape(T, P * C_))


class Comm:
    """An NCCL communicator on one CudaBackend context (tpt_cuda_comm_*)."""

    def __init__(self, be, handle, world, rank):
        self.be = be  # the context must outlive the communicator
        self.h = handle
        self.world = world
        self.rank = rank

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_ubyte * COMM_ID_BYTES)()
        st = lib.tpt_cuda_comm_unique_id(buf, COMM_ID_BYTES)
        if st != OK:
            raise OpError(st)
        return bytes(buf)

    @classmethod
    def create(cls, be, world: int, rank: int, broadcast):
        """``broadcast(obj_or_None) -> obj`` delivers rank 0's id to every rank."""
        uid = broadcast(cls.unique_id() if rank == 0 else None)
        buf = (C.c_ubyte * COMM_ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p()
        be._check(lib.tpt_cuda_comm_create(be.ctx, buf, COMM_ID_BYTES, world, rank, C.byref(h)))
        return cls(be, h, world, rank)

    def all_gather_dev(self, src, dst, bytes_per_rank: int):
        """dst [world * bytes] = every rank's src [bytes] (torch CUDA tensors), async."""
        self.be._check(lib.tpt_cuda_all_gather_dev(self.h, C.c_void_p(src.data_ptr()), C.c_void_p(dst.data_ptr()),
                                                   bytes_per_rank))

    def close(self):
        if self.h:
            lib.tpt_cuda_comm_destroy(self.h)
            self.h = None


def torch_broadcast(obj):
    """Rank 0's ``obj`` on every rank, over the default torch.distributed group."""
    import torch.distributed as dist

    box = [obj]
    dist.broadcast_object_list(box, src=0)
    return box[0]
