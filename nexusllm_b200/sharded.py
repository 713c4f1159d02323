"""Row-sharded GEMV stacks across the GPUs of one node (one process per GPU).

Host-side plumbing around nexus_gpu_stack_create_sharded / _export / _connect
(include/nexus_gpu.h).  The reference runs every GEMV of a decode step on one
device (src/forward_pass.cpp:504-585); here every rank owns the contiguous row
slice ``shard_rows(rows, world, rank)`` of every matrix, and the stack kernel
writes each rank's output rows straight into every peer's copy of the output
(the all-gather fused into the GEMV epilogue).  The only host exchange is the
CUDA IPC blobs, once, through a torch.distributed process group (gloo or nccl).
"""
from __future__ import annotations

import ctypes
from typing import Callable, Sequence

from . import _native


def shard_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of a ``rows``-row matrix owned by ``rank`` of ``world``
    (the same split the library makes)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    return rows * rank // world, rows * (rank + 1) // world


def exchange_blobs(blob: bytes, world: int, rank: int, all_gather: Callable | None = None) -> bytes:
    """Gather every rank's blob, concatenated in rank order.

    ``all_gather(obj) -> list`` defaults to torch.distributed.all_gather_object
    on the default group."""
    if all_gather is None:
        import torch.distributed as dist

        def all_gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

    got = all_gather((rank, bytes(blob)))
    if len(got) != world:
        raise RuntimeError(f"exchange returned {len(got)} blobs for {world} ranks")
    by_rank = dict(got)
    if sorted(by_rank) != list(range(world)):
        raise RuntimeError(f"exchange returned blobs of ranks {sorted(by_rank)}")
    return b"".join(by_rank[r] for r in range(world))


class ShardedStack:
    """A GEMV stack row-sharded over ``world`` GPUs.

    ``tasks``: sequence of (W_slice_ptr, rows, cols, x_source, after) with the
    FULL row count and this rank's row slice of W (``shard_rows``), as for
    nexus_gpu_stack_create_sharded; optionally followed by (x_source2,
    residual_source, norm_weight_ptr, norm_eps, W_up_slice_ptr), the fusions
    of nexus_gpu_stack_create_ex.  Outputs are full-length on every rank
    (``output(i)``)."""

    def __init__(self, dtype: int, tasks: Sequence[tuple], input_cols: int, world: int, rank: int,
                 all_gather: Callable | None = None, lib=None):
        self.L = lib if lib is not None else _native.lib()
        self.world, self.rank = world, rank
        arr = (_native.StackTaskEx * len(tasks))()
        for i, t in enumerate(tasks):
            w, rows, cols, src, after = t[:5]
            # optional fusions (nexus_gpu_stack_create_ex): x_source2, residual_source, norm
            # weights, eps, and this rank's row slice of the up matrix of a gate+up pair
            src2, res, nw, eps, w_up = tuple(t[5:]) + (-1, -2, None, 0.0, None)[len(t) - 5:]
            arr[i] = _native.StackTaskEx(w, rows, cols, None, src, after, src2, res, nw, eps, w_up)
        h = ctypes.c_void_p()
        _native.check(self.L.nexus_gpu_stack_create_ex(dtype, arr, len(tasks), input_cols, world, rank,
                                                        ctypes.byref(h)))
        self.handle = h
        try:
            size = ctypes.c_uint64(0)
            _native.check(self.L.nexus_gpu_stack_export(h, None, ctypes.byref(size)))
            buf = ctypes.create_string_buffer(size.value)
            _native.check(self.L.nexus_gpu_stack_export(h, buf, ctypes.byref(size)))
            blobs = exchange_blobs(buf.raw[:size.value], world, rank, all_gather)
            _native.check(self.L.nexus_gpu_stack_connect(h, blobs, len(blobs)))
        except Exception:
            self.close()
            raise

    def run(self, x_ptr: int, stream_ptr: int) -> None:
        _native.check(self.L.nexus_gpu_stack_run(self.handle, x_ptr, stream_ptr))

    def output(self, task: int) -> int:
        p = ctypes.c_void_p()
        _native.check(self.L.nexus_gpu_stack_output(self.handle, task, ctypes.byref(p)))
        return p.value

    def close(self) -> None:
        if self.handle is not None and self.handle.value:
            self.L.nexus_gpu_stack_destroy(self.handle)
        self.handle = None
