"""Benchmark: quantized GEMV HBM throughput and decode layer-stack tokens/s.

Workload (M=1): one decode token through a
Llama-3-8B-shaped Q4_0 stack -- 32 layers x {q 4096x4096, k 1024x4096,
v 1024x4096, o 4096x4096, gate 14336x4096, up 14336x4096, down 4096x14336}
plus the LM head 128256x4096 -- 225 fused GEMVs, 4.22 GB of weights, far
larger than L2 (so every step streams weights from HBM; no L2 flush needed).
Within a layer each GEMV consumes the previous one's output (q feeds o as a
stand-in for attention, o feeds gate and up, gate feeds down); every layer
starts from the same resident hidden state.  Weights are seeded synthetic
GGUF blocks with the configuration's distributions (nexusllm_b200/synth.py),
generated on the device.

A step = one token = the 225 GEMVs as ONE persistent GEMV-stack launch
(nexus_gpu_stack_run), captured once in a CUDA graph and replayed.  With
--gpus N > 1 (torchrun, one rank per GPU) every matrix is row-sharded over the
ranks and the stack kernel stores each rank's output rows straight into every
peer's output over NVLink (the all-gather fused into the GEMV; strong
scaling: the same model at every N).  The same step as 225 separate GEMV
launches (+ NCCL all-gathers at N > 1) is timed as a secondary figure and
must agree bit for bit.

Reported (one JSON line on rank 0):
  value     whole-job algorithmic GB/s = (weight + x + y bytes per step) x
            steps / device time (max over ranks)
  e2e       same metric through the library's C ABI with host buffers:
            pinned host hidden state in, host logits out, every step
            (N=1 also reports the reference-facing nexus_gpu_gemv_dispatch
            path, one synchronous host-pointer call per GEMV)
  roofline  the stack kernel (the only kernel of the step), algorithmic
            bytes per launch / CUDA-event time, against MEASURED_PEAKS.json
  cpu_baseline  NexusLLM's own AVX2 GEMV (oracle/_ref) on this host's cores
            over one decode layer

--impl reference times only the reference CPU path (rank 0), same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, KV, FFN, VOCAB, LAYERS = 4096, 1024, 14336, 128256, 32
MODEL = "8b"


def layer_shapes():
    return [("q", HIDDEN, HIDDEN), ("k", KV, HIDDEN), ("v", KV, HIDDEN), ("o", HIDDEN, HIDDEN),
            ("gate", FFN, HIDDEN), ("up", FFN, HIDDEN), ("down", HIDDEN, FFN)]


LAYER_SHAPES = layer_shapes()


def set_model(name):
    """--model 70b: BASELINE.json configs[4], Llama-3-70B shapes (hidden 8192,
    GQA k/v 1024x8192, FFN 28672, 80 layers, LM head 128256x8192)."""
    global HIDDEN, KV, FFN, VOCAB, LAYERS, LAYER_SHAPES, MODEL
    MODEL = name
    if name == "70b":
        HIDDEN, KV, FFN, VOCAB, LAYERS = 8192, 1024, 28672, 128256, 80
    LAYER_SHAPES = layer_shapes()
DTYPE = 7  # GGUF_Q4_0
NOMINAL_HBM_GBS = 8000.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ helpers
def q4_bytes(rows, cols):
    return rows * (cols // 32) * 18


def step_bytes(include_head=True, layers=None):
    b = 0
    for _, n, k in LAYER_SHAPES:
        b += q4_bytes(n, k) + 4 * k + 4 * n
    b *= LAYERS if layers is None else layers
    if include_head:
        b += q4_bytes(VOCAB, HIDDEN) + 4 * HIDDEN + 4 * VOCAB
    return b


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clock and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu = gpu_id  # nvidia-smi -i accepts an index or a GPU UUID
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": smax, "reasons": ["no samples"]}
        load = sorted(sm)[len(sm) // 2:]  # upper half: samples under load
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


# ------------------------------------------------------------ reference arm
def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def gpu_uuid(torch, local):
    try:
        u = str(torch.cuda.get_device_properties(local).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(local)


def time_reference_layer(reps: int, threads: int, min_seconds: float = 0.0):
    """NexusLLM's own GEMV (oracle/_ref, AVX2+FMA) over one decode layer's 7
    matrices; returns (GB/s, seconds per layer, kind, sample description)."""
    import numpy as np

    import oracle
    from nexusllm_b200 import synth

    if oracle.reference_available():
        lib, kind = oracle.reference(), "reference"
    else:  # the reference sources were not available at build time
        lib, kind = oracle.port(), "port"
    mats = []
    for i, (name, n, k) in enumerate(LAYER_SHAPES):
        W = synth.blocks_numpy(DTYPE, n, k, 3000 + i)
        x = synth.activations_numpy(1, k, 3100 + i)[0]
        mats.append((W, x, np.zeros(n, np.float32), n, k))
    layer_bytes = sum(q4_bytes(n, k) + 4 * k + 4 * n for _, n, k in LAYER_SHAPES)

    def run_layer():
        for W, x, y, n, k in mats:
            if kind == "reference":
                oracle.gemv_threaded(lib, DTYPE, W, x, y, n, k, threads)
            else:
                y[:] = lib.gemv(DTYPE, W, x, n, k)

    run_layer()  # warm-up (page-in)
    t = []
    start = time.perf_counter()
    while len(t) < reps or time.perf_counter() - start < min_seconds:
        t0 = time.perf_counter()
        run_layer()
        t.append(time.perf_counter() - t0)
    reps = len(t)
    sec = statistics.median(t)
    sample = (f"one Llama-3-8B Q4_0 decode layer (7 GEMVs, {layer_bytes / 1e6:.1f} MB of weights) x {reps}, "
              f"rows split over {threads} threads, each thread calling the unmodified reference function")
    return layer_bytes / sec / 1e9, sec, kind, sample


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = cpu_threads()
    reps = max(1, args.steps)
    for _ in range(args.warmup):
        pass
    gbs, sec, kind, sample = time_reference_layer(reps, threads)
    reps = max(reps, 1)
    tok_s = gbs * 1e9 / step_bytes()
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": reps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, reference=True),
        "tokens_per_s": round(tok_s, 6),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = "quant GEMV achieved HBM GB/s (% of 8 TB/s) & decode layer-stack tokens/s @1/2/4/8"


def workload_config(args, reference=False):
    if MODEL == "70b":
        head = {"workload": "configs[4]: Llama-3-70B Q4_0 decode stack (80 layers x q,k,v,o,gate,up,down + LM head "
                            "128256x8192), batch M=1, fp32 activations",
                "model": "Llama-3-70B shapes (hidden 8192, kv 1024, ffn 28672, vocab 128256)"}
    else:
        head = {"workload": "configs[3]: Llama-3-8B Q4_0 decode stack (32 layers x q,k,v,o,gate,up,down + LM head "
                            "128256x4096), batch M=1, fp32 activations",
                "model": "Llama-3-8B shapes (hidden 4096, kv 1024, ffn 14336, vocab 128256)"}
    gb = step_bytes() / 1e9
    return {
        **head,
        "weight_format": "GGUF Q4_0", "global_batch": 1, "gemvs_per_step": 7 * LAYERS + 1,
        "parallelism": "cpu" if reference else (f"row-shard x{args.gpus} + NCCL all-gather" if args.gpus > 1
                                                else "single GPU"),
        "l2": f"working set {gb:.2f} GB per step >> 126 MB L2 (no flush needed)",
    }


# -------------------------------------------------------------- our arm
def build_stack(torch, rank, world, n_layers):
    """Weights for this rank: every matrix's row slice [rank*n/W, (rank+1)*n/W)."""
    from nexusllm_b200 import synth

    layers = []
    for l in range(n_layers):
        mats = {}
        for i, (name, n, k) in enumerate(LAYER_SHAPES):
            nl = n // world
            mats[name] = synth.blocks_torch(DTYPE, nl, k, 1000 * 3 + 10 * l + i + 100000 * rank)
        layers.append(mats)
    head = synth.blocks_torch(DTYPE, VOCAB // world, HIDDEN, 1000 * 3 + 999 + 100000 * rank)
    return layers, head


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-formats", action="store_true",
                    help="skip the per-format GEMV timings (GGUF formats, INT4-AWQ, FP8-E4M3)")
    ap.add_argument("--no-gguf", action="store_true",
                    help="skip the GGUF file -> device upload measurement")
    ap.add_argument("--no-fused", action="store_true",
                    help="skip the decode stack with RMSNorm / SwiGLU / residual fused in")
    ap.add_argument("--no-batched", action="store_true",
                    help="skip the batched-decode points (M = 4, 16, 64 tokens per step)")
    ap.add_argument("--model", default="8b", choices=["8b", "70b"],
                    help="8b: configs[3] (the headline); 70b: configs[4], Llama-3-70B shapes")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder layers in the stack (the configuration's count by default; fewer only for "
                         "profiling runs)")
    args = ap.parse_args()
    set_model(args.model)
    if args.layers is None:
        args.layers = LAYERS
    if args.model == "70b":
        # the 70B configuration is the batch-1 sharded stack; batched points,
        # per-format timings and the host-weight path stay with the 8B headline
        args.no_batched = args.no_formats = args.no_fused = args.no_gguf = True
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"

    from nexusllm_b200 import _native
    from nexusllm_b200.backend import CUDABackend

    be = CUDABackend()
    L = _native.lib()
    dev = torch.device("cuda", local)
    layers, head = build_stack(torch, rank, world, args.layers)
    stream = torch.cuda.Stream(dev)
    h0 = torch.randn(HIDDEN, generator=torch.Generator(device=dev).manual_seed(5), device=dev)

    # activation buffers: full vectors (inputs) and this rank's output slices
    def buf(n):
        return torch.empty(n, dtype=torch.float32, device=dev)

    full = {"q": buf(HIDDEN), "k": buf(KV), "v": buf(KV), "o": buf(HIDDEN), "gate": buf(FFN), "up": buf(FFN),
            "down": buf(HIDDEN), "head": buf(VOCAB)}
    part = {k: buf(v.numel() // world) for k, v in full.items()}
    # one workspace, sized for the largest K, passed explicitly (never allocates during capture)
    ws_bytes = max(L.nexus_gpu_gemv_workspace_size(DTYPE, 1, 1, k) for _, _, k in LAYER_SHAPES)
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=dev)
    inputs_of = {"q": None, "k": None, "v": None, "o": "q", "gate": "o", "up": "o", "down": "gate"}
    pg = dist.group.WORLD if world > 1 else None

    def gemv(W, x, name):
        n_local = part[name].numel()
        k = x.numel()
        st = torch.cuda.current_stream(dev).cuda_stream
        rc = L.nexus_gpu_gemv_ws(W.data_ptr(), DTYPE, x.data_ptr(), 0, part[name].data_ptr(), 1, n_local, k,
                                 ws.data_ptr(), ws.numel(), st)
        if rc:
            _native.check(rc)
        if world > 1:
            dist.all_gather_into_tensor(full[name], part[name], group=pg)
            return full[name]
        return part[name]

    def step():
        for mats in layers:
            for name, _, _ in LAYER_SHAPES:
                src = inputs_of[name]
                x = h0 if src is None else out[src]
                out[name] = gemv(mats[name], x, name)
        out["head"] = gemv(head, h0, "head")

    out = {}
    with torch.cuda.stream(stream):
        for _ in range(2):
            step()  # eager warm-up before capture (also warms NCCL)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def timed(fn, iters):
        # graph.replay() launches on torch's current stream: make that `stream`
        # and record the events on it
        barrier()
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                fn()
            e1.record()
        torch.cuda.synchronize(dev)
        barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    sb = step_bytes(layers=args.layers)
    peak, peak_kind = load_peaks()
    n_gemvs = 7 * args.layers + 1

    if world == 1:
        # ---- headline: the whole step in ONE persistent kernel (GEMV stack)
        stack, stack_graph, ys = build_stack_graph(torch, L, _native, layers, head, h0, stream, dev)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                stack_graph.replay()
        with Clocks(gpu_uuid(torch, local)) as clk:
            ms = timed(stack_graph.replay, args.steps)
        clocks = clk.summary()
        check_status(L)
        # the stack must reproduce the per-GEMV path bit for bit (LM head and last layer)
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize(dev)
        check_against_per_gemv(torch, (("head", ys[-1]), ("down", ys[-2]), ("gate", ys[-4])), out, "stack")
        verify_head(torch, be, head, h0, ys[-1], world, rank)
        ms_step = ms / args.steps
        value = sb * args.steps / (ms / 1e3) / 1e9
        # secondary: the same step as 225 separately launched GEMVs in a CUDA graph
        reps = max(10, args.steps // 5)
        ms_graph = timed(graph.replay, reps) / reps
        per_gemv = {"ms_per_step": round(ms_graph, 4), "value": round(sb / (ms_graph / 1e3) / 1e9, 1),
                    "unit": "GB/s", "tokens_per_s": round(1e3 / ms_graph, 2),
                    "launches_per_step": 2 * n_gemvs}
        roofline = {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(value / peak, 4), "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                    "kernel": "gemv_stack_kernel<FmtQ4_0,2>: the step's 225 GEMVs in one cooperative launch",
                    "bytes_per_launch": sb, "avg_launch_us": round(ms_step * 1e3, 2),
                    "launch_note": "one launch per step, after a 28 KB counter reset (cudaMemsetAsync)",
                    "traffic": round(STACK_TRAFFIC_PER_ALG_BYTE * sb)}
        e2e = None if args.no_e2e else e2e_stack_host(torch, L, stack, h0, ys[-1], stream, dev, args, timed, sb)
        e2e_dispatch = None if (args.no_e2e or args.model == "70b") else e2e_host_api(torch, L, layers, head, h0,
                                                                                      args)
        launches = args.steps
        launches_note = f"1 gemv_stack_kernel per step x {args.steps} steps (plus one counter memset per step)"
        extra = {"per_gemv_graph": per_gemv, "e2e_per_gemv_dispatch": e2e_dispatch}
        if not args.no_batched:
            extra["batched_decode"] = batched_decode(torch, L, layers, head, stream, dev, timed, args, peak, stack)
        if not args.no_formats:
            extra["gguf_gemv"] = gguf_formats(torch, L, stream, dev, timed, peak)
            extra["int4_awq_fp8"] = other_formats(torch, L, stream, dev, timed, peak)
        if not args.no_fused:
            extra["fused_decode_stack"] = fused_decode_stack(torch, L, layers, head, h0, stream, dev, timed, args, peak)
        if not args.no_gguf:
            extra["gguf_upload"] = gguf_upload(torch, L, dev)
        del stack_graph
        L.nexus_gpu_stack_destroy(stack)
    else:
        # ---- headline: the row-sharded stack, all-gather fused into the kernel
        sst, sgraph, souts = build_sharded_stack_graph(torch, L, layers, head, h0, stream, dev, world, rank)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                sgraph.replay()
        with Clocks(gpu_uuid(torch, local)) as clk:
            ms = timed(sgraph.replay, args.steps)
        clocks = clk.summary()
        check_status(L)
        # bit-exact against the per-GEMV path with NCCL all-gathers
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize(dev)
        check_against_per_gemv(torch, (("head", souts[-1]), ("down", souts[-2]), ("gate", souts[-4])), out,
                               "sharded stack")
        ms_step = ms / args.steps
        value = sb * args.steps / (ms / 1e3) / 1e9
        reps = max(10, args.steps // 5)
        ms_graph = timed(graph.replay, reps) / reps
        per_gemv = {"ms_per_step": round(ms_graph, 4), "value": round(sb / (ms_graph / 1e3) / 1e9, 1),
                    "unit": "GB/s", "tokens_per_s": round(1e3 / ms_graph, 2),
                    "launches_per_step": 2 * n_gemvs, "nccl_all_gathers_per_step": n_gemvs}
        per_gpu = sb / world
        roofline = {"bound": "hbm", "achieved": round(per_gpu / (ms_step * 1e-3) / 1e9, 1), "peak": peak,
                    "unit": "GB/s", "frac": round(per_gpu / (ms_step * 1e-3) / 1e9 / peak, 4),
                    "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                    "kernel": f"gemv_stack_kernel<FmtQ4_0,2>, rank's 1/{world} row slice of every GEMV, "
                              "output rows stored into every peer over NVLink",
                    "bytes_per_launch": int(per_gpu), "avg_launch_us": round(ms_step * 1e3, 2),
                    "traffic": round(STACK_TRAFFIC_PER_ALG_BYTE * per_gpu)}
        e2e = None if args.no_e2e else e2e_sharded(torch, sst, sgraph, h0, souts[-1], stream, dev, args, timed, sb)
        launches = args.steps
        launches_note = (f"1 gemv_stack_kernel per step per GPU x {args.steps} steps; no NCCL in the step "
                         "(peer stores + peer counters inside the kernel)")
        extra = {"per_gemv_graph_nccl": per_gemv}
        del sgraph
        sst.close()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, sec, kind, sample = time_reference_layer(3, cpu_threads(), min_seconds=10.0)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cpu_threads(), "kind": kind, "sample": sample}

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8+fp32",
        "dtype_note": "Q4_0 codes x 16-bit fixed-point x in int8 dp4a limbs, fp32 accumulation",
        "data": "synthetic (seeded GGUF Q4_0 blocks, x ~ N(0,1))",
        "config": workload_config(args),
        "layers": args.layers,
        "pct_of_8tbs": round(100 * value / NOMINAL_HBM_GBS, 2),
        "pct_of_measured_hbm": round(100 * value / peak, 2),
        "tokens_per_s": round(1e3 / ms_step, 2),
        "gemv_calls_per_s": round(n_gemvs * 1e3 / ms_step, 1),
        "bytes_per_step": sb,
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
        "gpu_launches": launches, "gpu_launches_note": launches_note,
    }
    line.update(extra)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def check_against_per_gemv(torch, pairs, out, what):
    """The stack against the same GEMVs launched one by one: bit for bit where
    the task reads the stack input (the LM head), and within 1e-5 L2-relative
    where it reads another task's output (the stack hands a dependent task its
    source's output with the lowest mantissa bit cleared; the per-GEMV path
    passes the exact floats)."""
    for name, y in pairs:
        ref = out[name]
        if name == "head":
            ok = torch.equal(y, ref)
        else:
            ok = float(torch.linalg.vector_norm(y - ref) / torch.linalg.vector_norm(ref)) <= 1e-5
        if not ok:
            raise RuntimeError(f"{what} output of {name} differs from the per-GEMV path")


def check_status(L):
    import ctypes

    bits = ctypes.c_uint32(0)
    L.nexus_gpu_device_status(ctypes.byref(bits))
    if bits.value:
        raise RuntimeError(f"device status word {bits.value:#x} (a bounded wait expired)")


def batched_decode(torch, L, layers, head, stream, dev, timed, args, peak, stack=None):
    """configs[3] at M = 4, 16, 64 tokens per step (N=1): the step's 225
    GEMVs with M activation rows each, one nexus_gpu_gemv_ws call per GEMV,
    captured in a CUDA graph.  M >= 16 runs on the tcgen05 tensor cores; M = 4
    runs the batch-1 CUDA-core kernel once per token.  Same weights as the
    headline; a step reads every weight once per call."""
    out = []
    ws_need = 0
    for M in (4, 16, 64):
        ws_need = max([ws_need] + [L.nexus_gpu_gemv_workspace_size(DTYPE, M, n, k) for _, n, k in LAYER_SHAPES]
                      + [L.nexus_gpu_gemv_workspace_size(DTYPE, M, VOCAB, HIDDEN)])
    ws = torch.empty(ws_need + 256, dtype=torch.uint8, device=dev)
    for M in (4, 16, 64):
        xs = {k: torch.randn(M, k, generator=torch.Generator(device=dev).manual_seed(11 + k), device=dev)
              for k in (HIDDEN, FFN)}
        ys = {n: torch.empty(M, n, dtype=torch.float32, device=dev) for n in (HIDDEN, KV, FFN, VOCAB)}

        def step():
            st = torch.cuda.current_stream(dev).cuda_stream
            for mats in layers:
                for name, n, k in LAYER_SHAPES:
                    rc = L.nexus_gpu_gemv_ws(mats[name].data_ptr(), DTYPE, xs[k].data_ptr(), 0, ys[n].data_ptr(), M, n,
                                             k, ws.data_ptr(), ws.numel(), st)
                    if rc:
                        raise RuntimeError(L.nexus_gpu_last_error())
            rc = L.nexus_gpu_gemv_ws(head.data_ptr(), DTYPE, xs[HIDDEN].data_ptr(), 0, ys[VOCAB].data_ptr(), M, VOCAB,
                                     HIDDEN, ws.data_ptr(), ws.numel(), st)
            if rc:
                raise RuntimeError(L.nexus_gpu_last_error())

        with torch.cuda.stream(stream):
            step()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        with torch.cuda.stream(stream):
            for _ in range(3):
                g.replay()
        reps = max(5, min(50, args.steps // 20))
        ms = timed(g.replay, reps) / reps
        sb = step_bytes(layers=len(layers))
        gbs = sb / (ms * 1e-3) / 1e9
        out.append({"M": M, "ms_per_step": round(ms, 4), "tokens_per_s": round(M * 1e3 / ms, 1),
                    "value": round(gbs, 1), "unit": "GB/s", "pct_of_measured_hbm": round(100 * gbs / peak, 2),
                    "path": "tcgen05 kind::f16 (gemm_q4_0_mma_kernel)" if M >= 16 else
                            "batch-1 CUDA-core kernel per token", "steps": reps})
        del g
    if stack is not None:
        # M = 4 tokens through the GEMV stack, one launch per token (the batch-1
        # CUDA-core path, without per-GEMV launches); each token has its own
        # input, and each run overwrites the previous token's outputs (an engine
        # reads a token's logits before its next run)
        M = 4
        xs = [torch.randn(HIDDEN, generator=torch.Generator(device=dev).manual_seed(40 + m), device=dev)
              for m in range(M)]

        def step4():
            st = torch.cuda.current_stream(dev).cuda_stream
            for m in range(M):
                _native_check(L.nexus_gpu_stack_run(stack, xs[m].data_ptr(), st))

        with torch.cuda.stream(stream):
            step4()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step4()
        with torch.cuda.stream(stream):
            for _ in range(3):
                g.replay()
        reps = max(5, min(50, args.steps // 20))
        ms = timed(g.replay, reps) / reps
        gbs = step_bytes(layers=len(layers)) / (ms * 1e-3) / 1e9  # weights once per step, as above
        out.append({"M": M, "ms_per_step": round(ms, 4), "tokens_per_s": round(M * 1e3 / ms, 1),
                    "value": round(gbs, 1), "unit": "GB/s", "pct_of_measured_hbm": round(100 * gbs / peak, 2),
                    "path": "GEMV stack once per token (batch-1 CUDA-core path, one launch per token)",
                    "steps": reps})
        del g
    return out


def gguf_formats(torch, L, stream, dev, timed, peak):
    """Batch-1 GEMV per GGUF format (Q4_0, Q8_0, Q5_K, Q6_K, FP16) through
    nexus_gpu_gemv, the drop-in for the reference's fused_gemv_* (x quantized,
    then the fused GEMV: two launches a call), on the Llama-3-8B FFN and LM
    head shapes and the 70B FFN shapes.  Seeded blocks with the configs'
    distributions; each shape cycles over enough weight copies for >= 512 MB
    per graph pass (weights come from HBM); GB/s counts weights, x and y once
    per call."""
    from nexusllm_b200 import synth
    from nexusllm_b200.formats import weight_bytes

    shapes = [(14336, 4096), (4096, 14336), (128256, 4096), (28672, 8192), (8192, 28672)]
    out = []
    for dt, name in ((7, "q4_0"), (9, "q8_0"), (11, "q5_k"), (12, "q6_k"), (1, "fp16")):
        for rows, cols in shapes:
            wb = weight_bytes(dt, rows, cols)
            alg = wb + cols * 4 + rows * 4
            n = max(1, -(-(512 << 20) // wb))
            W = [synth.blocks_torch(dt, rows, cols, 4000 + 7 * i + dt) for i in range(n)]
            x = torch.randn(cols, device=dev, generator=torch.Generator(device=dev).manual_seed(cols))
            y = torch.empty(rows, device=dev)
            calls = 2 * n

            def run():
                st = torch.cuda.current_stream(dev).cuda_stream
                for i in range(calls):
                    rc = L.nexus_gpu_gemv(W[i % n].data_ptr(), dt, x.data_ptr(), 0, y.data_ptr(), 1, rows, cols, st)
                    if rc:
                        raise RuntimeError(L.nexus_gpu_last_error())

            with torch.cuda.stream(stream):
                run()
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                run()
            with torch.cuda.stream(stream):
                for _ in range(3):
                    g.replay()
            reps = 5
            ms = timed(g.replay, reps) / (reps * calls)
            gbs = alg / (ms * 1e-3) / 1e9
            out.append({"format": name, "rows": rows, "cols": cols, "us_per_call": round(ms * 1e3, 2),
                        "value": round(gbs, 1), "unit": "GB/s", "pct_of_measured_hbm": round(100 * gbs / peak, 1),
                        "gemv_calls_per_s": round(1e3 / ms, 1), "bytes_per_call": alg, "weight_copies": n})
            del g, W
    return out


def other_formats(torch, L, stream, dev, timed, peak):
    """INT4-AWQ (group 128, zeros) and FP8-E4M3 batch-1 GEMVs on the
    Llama-3-8B shapes, through nexus_gpu_gemv_int4 / nexus_gpu_gemv_fp8 (the
    reference's fused_gemv_int4 / fused_gemv_fp8).  Each shape cycles over
    enough weight copies for >= 512 MB per graph pass (weights come from HBM);
    GB/s counts weights, scales, zeros, x and y once per call."""
    shapes = [(HIDDEN, HIDDEN), (FFN, HIDDEN), (HIDDEN, FFN), (VOCAB, HIDDEN)]
    gs = 128
    out = []
    for fmt in ("int4_awq", "fp8_e4m3"):
        for rows, cols in shapes:
            if fmt == "int4_awq":
                wbytes = rows * cols // 2
                sbytes = 2 * rows * (cols // gs) * 4
            else:
                wbytes, sbytes = rows * cols, 0
            alg = wbytes + sbytes + cols * 4 + rows * 4
            n = max(1, -(-(512 << 20) // (wbytes + sbytes)))
            gen = torch.Generator(device=dev).manual_seed(rows + cols)
            if fmt == "int4_awq":
                W = [torch.randint(-2**31, 2**31 - 1, (rows * cols // 8,), dtype=torch.int32, device=dev,
                                   generator=gen) for _ in range(n)]
                S = [torch.rand(rows * cols // gs, device=dev, generator=gen) * 0.02 for _ in range(n)]
                Z = [torch.randint(0, 16, (rows * cols // gs,), device=dev, generator=gen).float() for _ in range(n)]
            else:  # realistic E4M3 codes (no NaN encodings)
                W = [(torch.randn(rows * cols, device=dev, generator=gen) * 0.5).to(torch.float8_e4m3fn).view(
                    torch.uint8) for _ in range(n)]
            x = torch.randn(cols, device=dev, generator=gen)
            y = torch.empty(rows, device=dev)
            calls = 2 * n

            def run():
                st = torch.cuda.current_stream(dev).cuda_stream
                for i in range(calls):
                    j = i % n
                    if fmt == "int4_awq":
                        rc = L.nexus_gpu_gemv_int4(W[j].data_ptr(), S[j].data_ptr(), Z[j].data_ptr(), x.data_ptr(),
                                                   y.data_ptr(), rows, cols, gs, None, 0, st)
                    else:
                        rc = L.nexus_gpu_gemv_fp8(W[j].data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, 0.0625, st)
                    if rc:
                        raise RuntimeError(L.nexus_gpu_last_error())

            with torch.cuda.stream(stream):
                run()
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                run()
            with torch.cuda.stream(stream):
                for _ in range(3):
                    g.replay()
            reps = 5
            ms = timed(g.replay, reps) / (reps * calls)
            gbs = alg / (ms * 1e-3) / 1e9
            out.append({"format": fmt, "rows": rows, "cols": cols, "group_size": gs if fmt == "int4_awq" else None,
                        "us_per_call": round(ms * 1e3, 2), "value": round(gbs, 1), "unit": "GB/s",
                        "pct_of_measured_hbm": round(100 * gbs / peak, 1), "bytes_per_call": alg,
                        "weight_copies": n})
            del g, W
            if fmt == "int4_awq":
                del S, Z
    return out


def fused_decode_stack(torch, L, layers, head, h0, stream, dev, timed, args, peak):
    """The same weights as the headline, with the reference decode layer's
    dataflow (src/forward_pass.cpp:504-562) fused into ONE stack launch:
    RMSNorm -> q, k, v; o (x = q, standing in for attention) + residual;
    RMSNorm -> gate+up pair with the SwiGLU epilogue; down + residual; final
    RMSNorm -> LM head (nexus_gpu_stack_create_ex, 6 tasks per layer).  Norm
    weights ~ 1 + N(0, 0.1^2)."""
    import ctypes

    from nexusllm_b200 import _native

    gen = torch.Generator(device=dev).manual_seed(77)
    norm = lambda: 1.0 + 0.1 * torch.randn(HIDDEN, device=dev, generator=gen)  # noqa: E731
    keep, tasks = [], []
    prev = -1
    eps = 1e-5
    for mats in layers:
        b = len(tasks)
        na, nf = norm(), norm()
        keep += [na, nf]
        spec = [("q", prev, -2, na, None), ("k", prev, -2, na, None), ("v", prev, -2, na, None),
                ("o", b, prev, None, None), ("gate", b + 3, -2, nf, "up"), ("down", b + 4, b + 3, None, None)]
        shapes = {name: (n, k) for name, n, k in LAYER_SHAPES}
        for name, src, res, nw, pair in spec:
            n, k = shapes[name]
            y = torch.empty(n, dtype=torch.float32, device=dev)
            keep.append(y)
            tasks.append(_native.StackTaskEx(mats[name].data_ptr(), n, k, y.data_ptr(), src, -1, -1, res,
                                             None if nw is None else nw.data_ptr(), eps,
                                             None if pair is None else mats[pair].data_ptr()))
        prev = b + 5
    no = norm()
    y = torch.empty(VOCAB, dtype=torch.float32, device=dev)
    keep += [no, y]
    tasks.append(_native.StackTaskEx(head.data_ptr(), VOCAB, HIDDEN, y.data_ptr(), prev, -1, -1, -2, no.data_ptr(), eps))
    arr = (_native.StackTaskEx * len(tasks))(*tasks)
    h = ctypes.c_void_p()
    _native.check(L.nexus_gpu_stack_create_ex(DTYPE, arr, len(tasks), HIDDEN, 1, 0, ctypes.byref(h)))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        _native.check(L.nexus_gpu_stack_run(h, h0.data_ptr(), stream.cuda_stream))
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g, stream=stream):
            _native.check(L.nexus_gpu_stack_run(h, h0.data_ptr(), stream.cuda_stream))
        for _ in range(3):
            g.replay()
    reps = max(20, min(300, args.steps))
    ms = timed(g.replay, reps) / reps
    check_status(L)
    if not bool(torch.isfinite(y).all()):
        raise RuntimeError("fused decode stack produced non-finite logits")
    sb = step_bytes(layers=len(layers)) + 4 * HIDDEN * (2 * len(layers) + 1)  # + norm weights
    gbs = sb / (ms * 1e-3) / 1e9
    del g
    L.nexus_gpu_stack_destroy(h)
    return {"ms_per_step": round(ms, 4), "tokens_per_s": round(1e3 / ms, 2), "value": round(gbs, 1), "unit": "GB/s",
            "pct_of_measured_hbm": round(100 * gbs / peak, 2), "steps": reps,
            "dataflow": "RMSNorm->q,k,v; o(x=q)+residual; RMSNorm->gate+up pair, SwiGLU epilogue; down+residual; "
                        "RMSNorm->head",
            "launches_per_step": 1}


def gguf_upload(torch, L, dev):
    """The GGUF load path: a Llama-3-8B-shaped Q4_0 GGUF file (token_embd,
    32 layers x 7 matrices, output; tensor data repeats one 64 MiB random
    block) is written to a temporary directory, parsed (nexus_gpu_gguf_open)
    and uploaded into one preallocated device image (nexus_gpu_gguf_upload:
    host threads fill pinned staging buffers from the mapping while the
    previous pieces copy).  The file was just written, so the page cache is
    warm.  Beside it: the pinned host-to-device copy rate (the link's
    ceiling) and per-tensor pageable copies from a numpy memmap of the file
    (the plain way: torch .to(device) per tensor)."""
    import ctypes
    import shutil
    import tempfile
    import time

    import numpy as np

    from nexusllm_b200 import _native, gguf

    # one ~64 MiB pattern of whole Q4_0 blocks (scales ~U[0.005, 0.02], random nibbles), repeated
    rng = np.random.default_rng(3)
    nbk = (64 << 20) // 18
    blk = np.empty((nbk, 18), np.uint8)
    blk[:, :2] = rng.uniform(0.005, 0.02, nbk).astype(np.float16).view(np.uint8).reshape(nbk, 2)
    blk[:, 2:] = rng.integers(0, 256, (nbk, 16), dtype=np.uint8)
    block = blk.tobytes()

    def filler(n):
        def fn(f):
            left = n
            while left:
                k = min(left, len(block))
                f.write(block[:k])
                left -= k
        return (n, fn)

    q4 = lambda rows, cols: filler(rows * cols // 32 * 18)  # noqa: E731
    tensors = [("token_embd.weight", gguf.GGML_Q4_0, [HIDDEN, VOCAB], q4(VOCAB, HIDDEN))]
    names = {"q": "attn_q", "k": "attn_k", "v": "attn_v", "o": "attn_output", "gate": "ffn_gate", "up": "ffn_up",
             "down": "ffn_down"}
    ones = np.ones(HIDDEN, np.float32).tobytes()
    for l in range(LAYERS):
        for name, n, k in LAYER_SHAPES:
            tensors.append((f"blk.{l}.{names[name]}.weight", gguf.GGML_Q4_0, [k, n], q4(n, k)))
        tensors += [(f"blk.{l}.attn_norm.weight", gguf.GGML_F32, [HIDDEN], ones),
                    (f"blk.{l}.ffn_norm.weight", gguf.GGML_F32, [HIDDEN], ones)]
    tensors += [("output_norm.weight", gguf.GGML_F32, [HIDDEN], ones),
                ("output.weight", gguf.GGML_Q4_0, [HIDDEN, VOCAB], q4(VOCAB, HIDDEN))]
    meta = [("general.architecture", gguf.STRING, "llama"), ("llama.embedding_length", gguf.U32, HIDDEN),
            ("llama.block_count", gguf.U32, LAYERS), ("llama.feed_forward_length", gguf.U32, FFN)]
    d = tempfile.mkdtemp(prefix="nexus_gguf_")
    path = os.path.join(d, "llama3-8b-q4_0.gguf")
    try:
        t0 = time.perf_counter()
        gguf.write_gguf(path, meta, tensors)
        write_s = time.perf_counter() - t0
        file_bytes = os.path.getsize(path)
        with gguf.GGUFFile(path) as f:
            idx = list(range(len(f.tensors)))
            arr = (ctypes.c_uint64 * len(idx))(*idx)
            offs = (ctypes.c_uint64 * len(idx))()
            size = L.nexus_gpu_gguf_upload_size(f._h, arr, len(idx))
            image = torch.empty(size, dtype=torch.uint8, device=dev)
            st = torch.cuda.current_stream(dev).cuda_stream
            times = []
            for _ in range(4):  # the first call also makes the staging ring
                torch.cuda.synchronize(dev)
                t0 = time.perf_counter()
                _native.check(L.nexus_gpu_gguf_upload(f._h, arr, len(idx), image.data_ptr(), size, offs, st))
                times.append(time.perf_counter() - t0)
            data_bytes = sum(t["bytes"] for t in f.tensors)
            # spot check: first and last tensor on the device equal the file
            mm = np.memmap(path, dtype=np.uint8, mode="r")
            for i in (0, len(idx) - 1):
                t = f.tensors[i]
                dev_bytes = image[offs[i]:offs[i] + 4096].cpu().numpy()
                if not np.array_equal(dev_bytes, mm[t["file_offset"]:t["file_offset"] + 4096]):
                    raise RuntimeError("GGUF upload produced wrong bytes")
            # plain per-tensor pageable copies
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            for t in f.tensors:
                torch.from_numpy(mm[t["file_offset"]:t["file_offset"] + t["bytes"]]).to(dev)
            torch.cuda.synchronize(dev)
            plain_s = time.perf_counter() - t0
            del mm
        # the decode step from this file: weights and norms uploaded once, one fused stack per token
        from nexusllm_b200.decode import GgufDecodeStack

        t0 = time.perf_counter()
        dec = GgufDecodeStack(path, device=dev)
        load_s = time.perf_counter() - t0
        xh = torch.randn(HIDDEN, device=dev, generator=torch.Generator(device=dev).manual_seed(1))
        sdec = torch.cuda.Stream(dev)
        with torch.cuda.stream(sdec):
            dec.step(xh, sdec)
        torch.cuda.synchronize(dev)
        gdec = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gdec, stream=sdec):
            dec.step(xh, sdec)
        with torch.cuda.stream(sdec):
            for _ in range(3):
                gdec.replay()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            ev[0].record()
            for _ in range(50):
                gdec.replay()
            ev[1].record()
        torch.cuda.synchronize(dev)
        dec_ms = ev[0].elapsed_time(ev[1]) / 50
        if not bool(torch.isfinite(dec.outputs[-1][1]).all()):
            raise RuntimeError("decode step from the GGUF file produced non-finite logits")
        del gdec
        dec.close()
        del dec
        host = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
        dbuf = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        dbuf.copy_(host, non_blocking=True)
        ev[0].record()
        for _ in range(3):
            dbuf.copy_(host, non_blocking=True)
        ev[1].record()
        torch.cuda.synchronize(dev)
        pinned_gbs = 3 * (1 << 30) / (ev[0].elapsed_time(ev[1]) * 1e-3) / 1e9
        del image, host, dbuf
    finally:
        shutil.rmtree(d, ignore_errors=True)
    best = min(times[1:])
    gbs = data_bytes / best / 1e9
    return {"file_bytes": file_bytes, "tensor_bytes": data_bytes,
            "tensors": len(tensors), "upload_s": round(best, 4), "upload_gbs": round(gbs, 2),
            "first_upload_s": round(times[0], 4), "pinned_h2d_gbs": round(pinned_gbs, 2),
            "frac_of_pinned_h2d": round(gbs / pinned_gbs, 3),
            "plain_per_tensor_pageable_gbs": round(data_bytes / plain_s / 1e9, 2),
            "write_file_s": round(write_s, 2), "page_cache": "warm (file just written)",
            "decode_from_file": {"load_s": round(load_s, 3), "ms_per_step": round(dec_ms, 4),
                                 "tokens_per_s": round(1e3 / dec_ms, 1),
                                 "path": "GgufDecodeStack: parse, upload, one fused stack (norms, gate+up pair, "
                                         "residuals) per token"}}


def build_stack_graph(torch, L, _native, layers, head, h0, stream, dev):
    """The step as one GEMV stack: per layer q, k, v (x = the hidden state,
    after the previous layer's down), o (x = q), gate, up (x = o), down
    (x = gate); then the LM head (x = the hidden state, after the last down).
    Captured once in a CUDA graph (counter reset + one launch)."""
    import ctypes

    tasks, ys = [], []
    inputs_of = {"q": -1, "k": -1, "v": -1, "o": 0, "gate": 3, "up": 3, "down": 4}
    last_down = -1
    for mats in layers:
        base = len(tasks)
        for i, (name, n, k) in enumerate(LAYER_SHAPES):
            y = torch.empty(n, dtype=torch.float32, device=dev)
            src = inputs_of[name]
            after = last_down if src < 0 else -1
            tasks.append(_native.StackTask(mats[name].data_ptr(), n, k, y.data_ptr(), src if src < 0 else base + src,
                                           after))
            ys.append(y)
        last_down = base + 6
    y = torch.empty(VOCAB, dtype=torch.float32, device=dev)
    tasks.append(_native.StackTask(head.data_ptr(), VOCAB, HIDDEN, y.data_ptr(), -1, last_down))
    ys.append(y)
    arr = (_native.StackTask * len(tasks))(*tasks)
    h = ctypes.c_void_p()
    _native.check(L.nexus_gpu_stack_create(DTYPE, arr, len(tasks), HIDDEN, ctypes.byref(h)))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        _native.check(L.nexus_gpu_stack_run(h, h0.data_ptr(), stream.cuda_stream))  # uncaptured warm run
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g, stream=stream):
            _native.check(L.nexus_gpu_stack_run(h, h0.data_ptr(), stream.cuda_stream))
    torch.cuda.synchronize(dev)
    return h, g, ys


def build_sharded_stack_graph(torch, L, layers, head, h0, stream, dev, world, rank):
    """This rank's row slices of the step's GEMVs as one sharded stack (same
    task order and dependencies as build_stack_graph); outputs are
    full-length on every rank.  Captured once in a CUDA graph."""
    from nexusllm_b200.sharded import ShardedStack

    tasks = []
    inputs_of = {"q": -1, "k": -1, "v": -1, "o": 0, "gate": 3, "up": 3, "down": 4}
    last_down = -1
    for mats in layers:
        base = len(tasks)
        for name, n, k in LAYER_SHAPES:
            src = inputs_of[name]
            tasks.append((mats[name].data_ptr(), n, k, src if src < 0 else base + src, last_down if src < 0 else -1))
        last_down = base + 6
    tasks.append((head.data_ptr(), VOCAB, HIDDEN, -1, last_down))
    st = ShardedStack(DTYPE, tasks, HIDDEN, world, rank)
    outs = []
    for i, (_, n, *_r) in enumerate(tasks):
        outs.append(torch.as_tensor(_DeviceVec(st.output(i), n), device=dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        st.run(h0.data_ptr(), stream.cuda_stream)  # uncaptured warm run (every rank runs it)
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g, stream=stream):
            st.run(h0.data_ptr(), stream.cuda_stream)
    torch.cuda.synchronize(dev)
    return st, g, outs


class _DeviceVec:
    """A library-owned fp32 device vector seen through __cuda_array_interface__."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 2}


def e2e_sharded(torch, st, sgraph, h0, y_head, stream, dev, args, timed, sb):
    """N > 1: per step, every rank copies the token's hidden state from pinned
    host memory, replays its sharded-stack graph, and copies the full logits
    back to pinned host memory (device-timed, max over ranks)."""
    hin = torch.empty(HIDDEN, dtype=torch.float32, pin_memory=True)
    hin.copy_(h0.cpu())
    hout = torch.empty(VOCAB, dtype=torch.float32, pin_memory=True)

    def one():
        h0.copy_(hin, non_blocking=True)
        sgraph.replay()
        hout.copy_(y_head, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(3):
            one()
        ms = timed(one, args.e2e_steps)
    return {"value": round(sb * args.e2e_steps / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": 4 * HIDDEN, "d2h_bytes_per_step": 4 * VOCAB,
            "ms_per_step": round(ms / args.e2e_steps, 4),
            "api": "sharded GEMV stack (nexus_gpu_stack_run) per rank; host hidden state in, host logits out "
                   "per step (device-timed, max over ranks)"}


def e2e_stack_host(torch, L, stack, h0, y_head, stream, dev, args, timed, sb):
    """The step through the library's public C ABI with host buffers: the
    token's hidden state is copied from pinned host memory
    (nexus_gpu_copy_host_to_device_async), the stack runs
    (nexus_gpu_stack_run), the logits are copied back to pinned host memory
    (nexus_gpu_copy_device_to_host_async), then the stream is synchronised --
    every step, inside the timed region."""
    import ctypes

    hin = torch.empty(HIDDEN, dtype=torch.float32, pin_memory=True)
    hin.copy_(h0.cpu())
    hout = torch.empty(VOCAB, dtype=torch.float32, pin_memory=True)
    xdev = torch.empty(HIDDEN, dtype=torch.float32, device=dev)
    st = ctypes.c_void_p(stream.cuda_stream)

    def one():
        _native_check(L.nexus_gpu_copy_host_to_device_async(xdev.data_ptr(), hin.data_ptr(), 4 * HIDDEN, st))
        _native_check(L.nexus_gpu_stack_run(stack, xdev.data_ptr(), st))
        _native_check(L.nexus_gpu_copy_device_to_host_async(hout.data_ptr(), y_head.data_ptr(), 4 * VOCAB, st))
        _native_check(L.nexus_gpu_synchronize(st))

    for _ in range(3):
        one()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        one()
    sec = (time.perf_counter() - t0) / args.e2e_steps
    torch.cuda.synchronize(dev)
    if not torch.equal(hout, y_head.cpu()):
        raise RuntimeError("host logits differ from the device result")
    return {"value": round(sb / sec / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": 4 * HIDDEN,
            "d2h_bytes_per_step": 4 * VOCAB, "ms_per_step": round(sec * 1e3, 4), "tokens_per_s": round(1 / sec, 2),
            "api": "nexus_gpu_copy_host_to_device_async + nexus_gpu_stack_run + "
                   "nexus_gpu_copy_device_to_host_async + nexus_gpu_synchronize, host wall clock per step",
            "steps": args.e2e_steps}


def _native_check(rc):
    from nexusllm_b200 import _native

    _native.check(rc)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per algorithmic
# byte of the stack kernel, from the ncu capture of a 4-layer Llama-3-8B Q4_0
# stack summarised in profiles/gemv_stack_q4_0_llama3_8b.md (traffic grows in
# proportion to the layers a launch processes).
STACK_TRAFFIC_PER_ALG_BYTE = (786439424 + 6302976) / 788075520  # 4 layers + LM head: read + written / algorithmic


def verify_head(torch, be, head, h0, y_graph, world, rank):
    """The replayed graph must have computed the LM head: compare this rank's
    slice (or, at N > 1, the gathered vector's slice) with an eager call."""
    torch.cuda.synchronize()
    y_eager = be.gemv(head, 7, h0)
    n = y_eager.numel()
    got = y_graph[rank * n:(rank + 1) * n] if world > 1 else y_graph[:n]
    if not torch.equal(got, y_eager):
        raise RuntimeError("graph replay did not reproduce the eager LM-head GEMV")


def e2e_host_api(torch, L, layers, head, h0, args):
    """The same step through the reference-facing C ABI: nexus_gpu_gemv_dispatch
    with HOST weights (cached on the device after the first call), host x and
    host y (pinned), one synchronous call per GEMV as the reference's forward
    pass makes them (src/forward_pass.cpp:504-585)."""
    import numpy as np

    host_layers = [{n: W.cpu().numpy() for n, W in mats.items()} for mats in layers]
    host_head = head.cpu().numpy()

    def pinned(n):
        return torch.empty(n, dtype=torch.float32, pin_memory=True).numpy()

    hx = pinned(HIDDEN)
    hx[:] = h0.cpu().numpy()
    outs = {"q": pinned(HIDDEN), "k": pinned(KV), "v": pinned(KV), "o": pinned(HIDDEN), "gate": pinned(FFN),
            "up": pinned(FFN), "down": pinned(HIDDEN), "head": pinned(VOCAB)}
    srcs = {"q": hx, "k": hx, "v": hx, "o": outs["q"], "gate": outs["o"], "up": outs["o"], "down": outs["gate"]}
    h2d = d2h = 0
    for _, n, k in LAYER_SHAPES:
        h2d += 4 * k
        d2h += 4 * n
    h2d = h2d * len(layers) + 4 * HIDDEN
    d2h = d2h * len(layers) + 4 * VOCAB

    def step():
        for hm in host_layers:
            for name, n, k in LAYER_SHAPES:
                rc = L.nexus_gpu_gemv_dispatch(hm[name].ctypes.data, DTYPE, srcs[name].ctypes.data,
                                               outs[name].ctypes.data, n, k)
                if rc:
                    raise RuntimeError(L.nexus_gpu_last_error())
        rc = L.nexus_gpu_gemv_dispatch(host_head.ctypes.data, DTYPE, hx.ctypes.data, outs["head"].ctypes.data,
                                       VOCAB, HIDDEN)
        if rc:
            raise RuntimeError(L.nexus_gpu_last_error())

    for _ in range(3):
        step()  # first call uploads every weight into the device cache
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        step()
    sec = (time.perf_counter() - t0) / args.e2e_steps
    L.nexus_gpu_weight_cache_invalidate(None)
    del host_layers, host_head
    return {"value": round(step_bytes(layers=len(layers)) / sec / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(sec * 1e3, 3), "tokens_per_s": round(1 / sec, 2),
            "api": "nexus_gpu_gemv_dispatch (host pointers, synchronous, weights cached on device)",
            "steps": args.e2e_steps}


if __name__ == "__main__":
    main()
