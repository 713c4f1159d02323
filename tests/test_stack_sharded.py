"""Host logic of row-sharded GEMV stacks, on the CPU.

Covers the row split, the blob exchange over a real two-rank gloo process
group, and the library's argument checks (which run before any device call).
The kernel itself is exercised on two GPUs by tests/test_stack_sharded_gpu.py.
"""
import ctypes
import socket

import pytest

from nexusllm_b200 import _native
from nexusllm_b200.sharded import exchange_blobs, shard_rows

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("rows", [1024, 4096, 14336, 128256, 3000, 1057, 8])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_partition(rows, world):
    spans = [shard_rows(rows, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == rows
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0  # contiguous, in rank order
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1  # balanced


def test_shard_rows_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_rows(100, 2, 2)
    with pytest.raises(ValueError):
        shard_rows(100, 0, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        blob = bytes([rank]) * (10 + rank)  # ranks' blobs differ in content and length
        got = exchange_blobs(blob, world, rank)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_exchange_blobs_two_gloo_ranks():
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = bytes([0]) * 10 + bytes([1]) * 11
    assert res[0] == want and res[1] == want  # every rank gets all blobs in rank order


def test_exchange_blobs_rejects_missing_rank():
    with pytest.raises(RuntimeError):
        exchange_blobs(b"x", 2, 0, all_gather=lambda obj: [obj, obj])  # rank 0 twice, rank 1 missing
    with pytest.raises(RuntimeError):
        exchange_blobs(b"x", 2, 0, all_gather=lambda obj: [obj])


def test_sharded_create_argument_checks():
    L = _native.lib()
    T = _native.StackTask
    arr = (T * 1)(T(16, 64, 64, None, -1, -1))
    h = ctypes.c_void_p()
    # world and rank are checked before any device is touched
    bad = -9  # NEXUS_GPU_ERROR_INVALID_ARGUMENT
    assert L.nexus_gpu_stack_create_sharded(7, arr, 1, 64, 1, 0, ctypes.byref(h)) == bad
    assert L.nexus_gpu_stack_create_sharded(7, arr, 1, 64, 9, 0, ctypes.byref(h)) == bad
    assert L.nexus_gpu_stack_create_sharded(7, arr, 1, 64, 2, 2, ctypes.byref(h)) == bad
    assert h.value is None
    size = ctypes.c_uint64(0)
    assert L.nexus_gpu_stack_export(None, None, ctypes.byref(size)) == bad
    assert L.nexus_gpu_stack_connect(None, b"", 0) == bad
    p = ctypes.c_void_p()
    assert L.nexus_gpu_stack_output(None, 0, ctypes.byref(p)) == bad


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_sharded_stack_without_device_fails_loudly():
    from nexusllm_b200.sharded import ShardedStack

    with pytest.raises(_native.NexusGpuError):
        ShardedStack(7, [(16, 64, 64, -1, -1)], 64, 2, 0, all_gather=lambda obj: [obj, (1, obj[1])])
