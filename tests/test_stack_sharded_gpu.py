"""Row-sharded GEMV stacks on two GPUs (skipped with fewer).

Two processes (one per GPU, gloo for the blob exchange) each own a row slice
of every matrix.  Every output of the sharded stack, on both ranks, must equal
the unsharded stack on the full matrices bit for bit: per-row arithmetic does
not depend on the split.  Runs again with a new input and under a CUDA graph
(counters are cumulative across runs, so no reset may be needed).  The fused
case adds the decode layer's RMSNorms, gate+up pairs with the SwiGLU epilogue
and residual adds (nexus_gpu_stack_create_ex): the norm reads the gathered
full-length input on every rank, so the split changes nothing there either.
"""
import socket

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spec(hidden, kv, ffn, layers, head_rows):
    out, last_down = [], -1
    for _ in range(layers):
        b = len(out)
        out += [(hidden, hidden, -1, last_down), (kv, hidden, -1, last_down), (kv, hidden, -1, last_down),
                (hidden, hidden, b + 0, -1), (ffn, hidden, b + 3, -1), (ffn, hidden, b + 3, -1),
                (hidden, ffn, b + 4, -1)]
        last_down = b + 6
    out.append((head_rows, hidden, -1, last_down))
    return out


def _fused_spec(hidden, kv, ffn, layers, head_rows):
    """(rows, cols, src, after, residual_source, norm?, pair?) of a fused decoder."""
    out, prev = [], -1
    for _ in range(layers):
        b = len(out)
        out += [(hidden, hidden, prev, -1, -2, True, False), (kv, hidden, prev, -1, -2, True, False),
                (kv, hidden, prev, -1, -2, True, False), (hidden, hidden, b + 0, -1, prev, False, False),
                (ffn, hidden, b + 3, -1, -2, True, True), (hidden, ffn, b + 4, -1, b + 3, False, False)]
        prev = b + 5
    out.append((head_rows, hidden, prev, -1, -2, True, False))
    return out


def _worker(rank, port, dt, dims, q, fused=False):
    import ctypes

    import torch
    import torch.distributed as dist

    from nexusllm_b200 import _native, synth
    from nexusllm_b200.formats import row_bytes
    from nexusllm_b200.sharded import ShardedStack, shard_rows

    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
        L = _native.lib()
        spec = _fused_spec(*dims) if fused else [t + (-2, False, False) for t in _spec(*dims)]
        hidden = spec[0][1]
        keep, tasks, arr, ref = [], [], (_native.StackTaskEx * len(spec))(), []
        g = torch.Generator().manual_seed(3)

        def slice_of(W, rows, cols):
            r0, r1 = shard_rows(rows, WORLD, rank)
            Wl = W.view(rows, row_bytes(dt, cols))[r0:r1].contiguous()
            keep.append(Wl)
            return Wl.data_ptr()

        for i, (rows, cols, src, after, res, norm, pair) in enumerate(spec):
            W = synth.blocks_torch(dt, rows, cols, 500 + i)  # the same bytes on every rank
            Wu = synth.blocks_torch(dt, rows, cols, 900 + i) if pair else None
            nw = (1.0 + 0.1 * torch.randn(cols, generator=g)).cuda() if norm else None
            keep += [W, Wu, nw]
            nwp = None if nw is None else nw.data_ptr()
            tasks.append((slice_of(W, rows, cols), rows, cols, src, after, -1, res, nwp, 1e-5,
                          slice_of(Wu, rows, cols) if pair else None))
            y = torch.empty(rows, device="cuda")  # the unsharded stack on this GPU, full matrices
            ref.append(y)
            arr[i] = _native.StackTaskEx(W.data_ptr(), rows, cols, y.data_ptr(), src, after, -1, res, nwp, 1e-5,
                                         None if Wu is None else Wu.data_ptr())
        st = ShardedStack(dt, tasks, hidden, WORLD, rank)
        h1 = ctypes.c_void_p()
        _native.check(L.nexus_gpu_stack_create_ex(dt, arr, len(spec), hidden, 1, 0, ctypes.byref(h1)))

        ptrs = [st.output(i) for i in range(len(spec))]
        stream = torch.cuda.Stream()
        bad = []
        for rep, seed in enumerate((11, 12, 11)):
            x = torch.from_numpy(synth.activations_numpy(1, hidden, seed)[0]).cuda()
            with torch.cuda.stream(stream):
                st.run(x.data_ptr(), stream.cuda_stream)
                _native.check(L.nexus_gpu_stack_run(h1, x.data_ptr(), stream.cuda_stream))
            torch.cuda.synchronize()
            for i, (rows, *_r) in enumerate(spec):
                got = torch.as_tensor(_DeviceArray(ptrs[i], rows), device="cuda").clone()
                if not torch.equal(got, ref[i]):
                    bad.append((rep, i))
            torch.cuda.synchronize()
            # a peer's next run writes into this rank's outputs: every rank
            # reads a run's outputs before any rank starts the next run
            dist.barrier()
        # under a CUDA graph: replays keep advancing the run counter on the device
        # (same input every replay, so outputs stay valid while peers run ahead)
        graph = torch.cuda.CUDAGraph()
        x = torch.from_numpy(synth.activations_numpy(1, hidden, 13)[0]).cuda()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph, stream=stream):
                st.run(x.data_ptr(), stream.cuda_stream)
            for _ in range(3):
                graph.replay()
            _native.check(L.nexus_gpu_stack_run(h1, x.data_ptr(), stream.cuda_stream))
        torch.cuda.synchronize()
        for i, (rows, *_r) in enumerate(spec):
            got = torch.as_tensor(_DeviceArray(ptrs[i], rows), device="cuda").clone()
            if not torch.equal(got, ref[i]):
                bad.append(("graph", i))
        bits = ctypes.c_uint32(0)
        L.nexus_gpu_device_status(ctypes.byref(bits))
        dist.barrier()
        del graph
        st.close()
        L.nexus_gpu_stack_destroy(h1)
        dist.destroy_process_group()
        q.put((rank, bad, bits.value, None))
    except Exception as e:  # report, never hang the parent
        q.put((rank, None, None, repr(e)))


class _DeviceArray:
    """A raw fp32 device vector exposed through __cuda_array_interface__."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 2}


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason=f"needs {WORLD} GPUs")
@pytest.mark.parametrize("dt,dims,fused", [(7, (2048, 512, 5632, 2, 3000), False),
                                           (12, (2048, 512, 5632, 2, 3000), False),
                                           (7, (4096, 1024, 14336, 1, 4099), False),
                                           (7, (2048, 512, 5632, 2, 3000), True),
                                           (7, (4096, 1024, 14336, 1, 4099), True)])
def test_sharded_stack_equals_unsharded(dt, dims, fused):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, dt, dims, q, fused)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            rank, bad, status, err = q.get(timeout=240)
            res[rank] = (bad, status, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank in range(WORLD):
        bad, status, err = res[rank]
        assert err is None, f"rank {rank}: {err}"
        assert status == 0, f"rank {rank}: device status {status:#x}"
        assert not bad, f"rank {rank}: outputs differ from the unsharded stack at {bad[:8]}"
