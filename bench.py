"""Benchmark: quantized GEMV HBM throughput and decode layer-stack tokens/s.

Headline (M=1): one decode token through a
Llama-3-8B-shaped Q4_0 stack -- 32 layers x {q 4096x4096, k 1024x4096,
v 1024x4096, o 4096x4096, gate 14336x4096, up 14336x4096, down 4096x14336}
plus the LM head 128256x4096 -- 225 fused GEMVs, 4.23 GB of weights, far
larger than L2 (every step streams weights from HBM; no L2 flush needed).
Within a layer each GEMV consumes the previous one's output (q feeds o as a
stand-in for attention, o feeds gate and up, gate feeds down); every layer
starts from the same resident hidden state.  Weights are seeded synthetic
GGUF blocks with the configuration's distributions, generated on the device
in 8 row blocks per matrix seeded by (matrix, block), so every GPU count runs
the same model byte for byte.

A step = one token = the 225 GEMVs as ONE persistent GEMV-stack launch
(nexus_gpu_stack_run), captured once in a CUDA graph and replayed.  With
--gpus N > 1 (torchrun, one rank per GPU) every matrix is row-sharded over the
ranks and the stack kernel stores each rank's output rows straight into every
peer's output over NVLink (the all-gather fused into the GEMV; strong
scaling).  Sampled rows of four tasks are checked against the C oracle (the
checker) at every N; the step as 225 separate launches (+ NCCL all-gathers
at N > 1) is timed as a secondary figure.

One JSON line on rank 0: the contract's keys (value = whole-job algorithmic
GB/s over device time, max over ranks; e2e through the C ABI with host
buffers; roofline of the stack kernel against MEASURED_PEAKS.json;
cpu_baseline = NexusLLM's own AVX2 GEMV over the whole step on this host),
then compact secondary tables, then -- last, so that a truncated log keeps
them -- the BASELINE configurations:
  config0_q4_0_4096         configs[0], per call and as a 64-GEMV stack, + CPU
  config1_q8_0_llama2_7b    configs[1], per shape, the set, the 32-layer stack, + CPU
  config2_q5k_q6k_llama2_7b configs[2], the Q5_K and Q6_K 32-layer stacks, + CPU
  model_70b                 configs[4] at this N: batch 1 (stack) and 16 (tcgen05)
(CPU legs: 1 thread and all host threads; "ms" is per call, per set, or per
token = 32 x one layer for configs[2].)

--impl reference times NexusLLM's own CPU GEMV over the whole step (rank 0).
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


class CpuStep:
    """The configs[3] decode step (32 layers x 7 GEMVs + LM head, 225 GEMVs,
    4.23 GB of Q4_0) on the host cores: NexusLLM's own fused_gemv_q4_0
    (oracle/_ref: src/quantization.cpp compiled unmodified, AVX2+FMA), or the
    C restatement where the reference build is absent.  Rows are split over
    `threads` host threads, each calling the unmodified reference function
    (Q4_0 has no OpenMP pragma in the reference, src/quantization.cpp:264-330,
    so it would otherwise use one core).  The layers cycle over DISTINCT
    weight buffers (about 0.5 GB, more than any host cache) and the LM head.
    Inputs are fixed seeded vectors; the timing does not depend on values."""

    DISTINCT = 4

    def __init__(self, m=None):
        import numpy as np

        import oracle
        from nexusllm_b200 import synth

        self.m = m or model_dims("8b")
        if oracle.reference_available():
            self.lib, self.kind = oracle.reference(), "reference"
        else:  # the reference sources were not available at build time
            self.lib, self.kind = oracle.port(), "port"
        shapes = shapes_of(self.m)
        base = [synth.blocks_numpy(DTYPE, n, k, 3000 + i) for i, (_, n, k) in enumerate(shapes)]
        self.layers = [[(np.copy(W), n, k) for W, (_, n, k) in zip(base, shapes)] for _ in range(self.DISTINCT)]
        self.head = (synth.blocks_numpy(DTYPE, self.m["vocab"], self.m["hidden"], 3999), self.m["vocab"],
                     self.m["hidden"])
        self.x = {k: synth.activations_numpy(1, k, 3100 + k)[0] for k in {k for _, _, k in shapes}}
        self.y = {n: np.zeros(n, np.float32) for n in {n for _, n, _ in shapes} | {self.m["vocab"]}}

    def gemv(self, W, n, k, threads):
        import oracle

        if self.kind == "reference":
            oracle.gemv_threaded(self.lib, DTYPE, W, self.x[k], self.y[n], n, k, threads)
        else:
            self.y[n][:] = self.lib.gemv(DTYPE, W, self.x[k], n, k)

    def run(self, threads):
        for l in range(self.m["layers"]):
            for W, n, k in self.layers[l % self.DISTINCT]:
                self.gemv(W, n, k, threads)
        self.gemv(*self.head, threads)

    def time(self, threads, reps, warmup, min_seconds=0.0):
        """Median seconds per step over >= reps steps (and >= min_seconds)."""
        for _ in range(warmup):
            self.run(threads)
        t, start = [], time.perf_counter()
        while len(t) < reps or time.perf_counter() - start < min_seconds:
            t0 = time.perf_counter()
            self.run(threads)
            t.append(time.perf_counter() - t0)
        return statistics.median(t), len(t)

    def sample(self, threads, steps, warmup):
        return (f"the whole configs[3] decode step ({7 * self.m['layers'] + 1} Q4_0 GEMVs incl. the LM head, "
                f"{model_bytes(self.m) / 1e9:.2f} GB) x {steps} steps after {warmup} warm-up steps, rows split over "
                f"{threads} threads each calling the unmodified reference fused_gemv_q4_0; layers cycle over "
                f"{self.DISTINCT} distinct weight buffers")


def run_reference(args):
    """--impl reference: NexusLLM's own CPU GEMV on this host's cores, the whole
    decode step per step (rank 0 only; other ranks exit without work)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = cpu_threads()
    reps = max(1, min(args.steps, 30))       # a whole step is ~0.3 s: bounded sample
    warmup = max(1, min(args.warmup, 10))
    step = CpuStep(model_dims(MODEL))
    sec, reps = step.time(threads, reps, warmup)
    sb = model_bytes(step.m)
    gbs = sb / sec / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": reps, "warmup": warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, reference=True),
        "tokens_per_s": round(1.0 / sec, 4),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": step.kind,
                         "sample": step.sample(threads, reps, warmup)},
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
        "parallelism": "cpu" if reference else (f"row-shard x{args.gpus}, all-gather fused into the GEMV stack "
                                                "(peer stores over NVLink)" if args.gpus > 1 else "single GPU"),
        "same_model_every_n": "weights seeded by global row (8 row blocks per matrix)",
        "l2": f"working set {gb:.2f} GB per step >> 126 MB L2 (no flush needed)",
    }


# -------------------------------------------------------------- our arm
# Every matrix is generated as CHUNKS row blocks, block c from seed (matrix
# seed, c): rank r of W (W in 1, 2, 4, 8) generates blocks [8r/W, 8(r+1)/W),
# which are exactly its rows [N*r/W, N*(r+1)/W).  So every N runs the SAME
# model, byte for byte.
CHUNKS = 8


def slice_blocks(torch, dt, N, K, seed, rank, world, dev):
    """Rank `rank`'s row slice of the seeded N x K matrix `seed` (GGUF blocks,
    flat uint8 on `dev`)."""
    from nexusllm_b200 import synth
    from nexusllm_b200.formats import weight_bytes

    assert N % CHUNKS == 0 and CHUNKS % world == 0, (N, world)
    c0, c1 = CHUNKS * rank // world, CHUNKS * (rank + 1) // world
    cb = weight_bytes(dt, N // CHUNKS, K)
    out = torch.empty((c1 - c0) * cb, dtype=torch.uint8, device=dev)
    for c in range(c0, c1):
        out[(c - c0) * cb:(c - c0 + 1) * cb].copy_(synth.blocks_torch(dt, N // CHUNKS, K, seed * 64 + c, device=dev))
    return out


def model_dims(name):
    """BASELINE configs[3] (8b) and configs[4] (70b) shapes."""
    if name == "70b":
        return {"name": "70b", "hidden": 8192, "kv": 1024, "ffn": 28672, "vocab": 128256, "layers": 80}
    return {"name": "8b", "hidden": 4096, "kv": 1024, "ffn": 14336, "vocab": 128256, "layers": 32}


def shapes_of(m):
    h, kv, f = m["hidden"], m["kv"], m["ffn"]
    return [("q", h, h), ("k", kv, h), ("v", kv, h), ("o", h, h), ("gate", f, h), ("up", f, h), ("down", h, f)]


def model_bytes(m, layers=None, dt=7):
    from nexusllm_b200.formats import weight_bytes

    b = sum(weight_bytes(dt, n, k) + 4 * k + 4 * n for _, n, k in shapes_of(m))
    return b * (m["layers"] if layers is None else layers) + weight_bytes(dt, m["vocab"], m["hidden"]) + \
        4 * m["hidden"] + 4 * m["vocab"]


def gen_model(torch, m, rank, world, dev, seed_base, n_layers=None, dt=7):
    """This rank's row slices of every matrix of model m (same bytes at every N)."""
    layers = []
    for l in range(m["layers"] if n_layers is None else n_layers):
        layers.append({name: slice_blocks(torch, dt, n, k, seed_base + 10 * l + i, rank, world, dev)
                       for i, (name, n, k) in enumerate(shapes_of(m))})
    head = slice_blocks(torch, dt, m["vocab"], m["hidden"], seed_base + 9999, rank, world, dev)
    return layers, head


def build_stack(torch, rank, world, n_layers):
    """Weights of the headline model for this rank (configs[3], seeded by global row)."""
    return gen_model(torch, model_dims(MODEL), rank, world, torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))),
                     3000, n_layers)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
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
    ap.add_argument("--no-configs", action="store_true",
                    help="skip BASELINE configs[0..2] (N=1) and the configs[4] Llama-3-70B object (every N)")
    ap.add_argument("--model", default="8b", choices=["8b", "70b"],
                    help="8b: configs[3] (the headline); 70b: configs[4] as the headline (profiling)")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder layers in the stack (the configuration's count by default; fewer only for "
                         "profiling runs)")
    args = ap.parse_args()
    set_model(args.model)
    if args.layers is None:
        args.layers = LAYERS
    if args.model == "70b":
        args.no_batched = args.no_formats = args.no_fused = args.no_gguf = args.no_configs = True
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
    extra, tail = {}, {}

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
        # the stack against the per-GEMV path (LM head bit for bit), and sampled rows against the oracle
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize(dev)
        check_against_per_gemv(torch, (("head", ys[-1]), ("down", ys[-2]), ("gate", ys[-4])), out, "stack")
        verify_head(torch, be, head, h0, ys[-1], world, rank)
        par = stack_parity(torch, layers, head, ys, h0, world, rank, dev)
        ms_step = ms / args.steps
        value = sb * args.steps / (ms / 1e3) / 1e9
        # secondary: the same step as 225 separately launched GEMVs in a CUDA graph
        reps = max(10, min(args.steps // 5, 50))
        ms_graph = timed(graph.replay, reps) / reps
        per_gemv = {"ms_per_step": round(ms_graph, 4), "GBs": round(sb / (ms_graph / 1e3) / 1e9, 1),
                    "launches_per_step": 2 * n_gemvs}
        roofline = {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(value / peak, 4), "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                    "kernel": "gemv_stack_kernel<FmtQ4_0,2>: the step's 225 GEMVs in one cooperative launch",
                    "bytes_per_launch": sb, "avg_launch_us": round(ms_step * 1e3, 2),
                    "traffic": round(STACK_TRAFFIC_PER_ALG_BYTE * sb)}
        e2e = None if args.no_e2e else e2e_stack_host(torch, L, stack, h0, ys[-1], stream, dev, args, timed, sb)
        e2e_dispatch = None if (args.no_e2e or args.model == "70b") else e2e_host_api(torch, L, layers, head, h0,
                                                                                      args)
        launches = args.steps
        launches_note = f"1 gemv_stack_kernel per step x {args.steps} steps"
        extra["per_gemv_graph"] = per_gemv
        if e2e_dispatch:
            extra["e2e_per_gemv_dispatch"] = {k: e2e_dispatch[k] for k in ("value", "unit", "ms_per_step")}
        if not args.no_batched:
            extra["batched_decode"] = batched_decode(torch, L, layers, head, stream, dev, timed, args, peak, stack)
        if not args.no_formats:
            extra["formats_gemv"] = gguf_formats(torch, L, stream, dev, timed, peak)
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
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize(dev)
        check_against_per_gemv(torch, (("head", souts[-1]), ("down", souts[-2]), ("gate", souts[-4])), out,
                               "sharded stack")
        par = stack_parity(torch, layers, head, souts, h0, world, rank, dev)
        ms_step = ms / args.steps
        value = sb * args.steps / (ms / 1e3) / 1e9
        reps = max(10, min(args.steps // 5, 50))
        ms_graph = timed(graph.replay, reps) / reps
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
                         "(peer stores inside the kernel)")
        extra["per_gemv_graph_nccl"] = {"ms_per_step": round(ms_graph, 4),
                                        "GBs": round(sb / (ms_graph / 1e3) / 1e9, 1),
                                        "launches_per_step": 2 * n_gemvs, "nccl_all_gathers_per_step": n_gemvs}
        del sgraph
        sst.close()
    del graph
    extra["parity"] = par

    # BASELINE configs[0..2] (one GPU) and configs[4] (every N), placed last in the line
    if not args.no_configs:
        del layers, head
        torch.cuda.empty_cache()
        if world == 1:
            tail["config0_q4_0_4096"] = config0(torch, L, dev, timed, peak)
            tail["config1_q8_0_llama2_7b"] = config1(torch, L, dev, timed, peak)
            tail["config2_q5k_q6k_llama2_7b"] = config2(torch, L, dev, timed, peak)
        tail["model_70b"] = model_70b(torch, L, world, rank, local, dev, timed, peak, args, pg)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cstep = CpuStep(model_dims(MODEL))
        threads = cpu_threads()
        sec, n = cstep.time(threads, 3, 1, min_seconds=10.0)
        cpu = {"value": round(model_bytes(cstep.m) / sec / 1e9, 3), "unit": "GB/s", "cores": threads,
               "kind": cstep.kind, "ms_per_step": round(sec * 1e3, 2), "sample": cstep.sample(threads, n, 1)}

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8+fp32",
        "dtype_note": "Q4_0 codes x 16-bit fixed-point x (exact int32 dp2a), fp32 scales and accumulation",
        "data": "synthetic (seeded GGUF Q4_0 blocks, x ~ N(0,1))",
        "config": workload_config(args),
        "layers": args.layers,
        "pct_of_measured_hbm": round(100 * value / peak, 2),
        "tokens_per_s": round(1e3 / ms_step, 2),
        "gemv_calls_per_s": round(n_gemvs * 1e3 / ms_step, 1),
        "bytes_per_step": sb,
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
        "gpu_launches": launches, "gpu_launches_note": launches_note,
    }
    line.update(extra)
    line.update(tail)
    if rank == 0:
        print(json.dumps(line, separators=(",", ":")), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def stack_parity(torch, layers, head, outs, h0, world, rank, dev):
    """Sampled rows of this rank's slice of the headline stack's first q, first
    o, last down and LM head against the C oracle, each task with the input the
    stack gave it; max over ranks."""
    import torch.distributed as dist

    from nexusllm_b200.formats import weight_bytes

    per = 7
    checks = [(layers[0]["q"], HIDDEN, HIDDEN, None, 0), (layers[0]["o"], HIDDEN, HIDDEN, 0, 3),
              (layers[-1]["down"], HIDDEN, FFN, per * (len(layers) - 1) + 4, per * (len(layers) - 1) + 6),
              (head, VOCAB, HIDDEN, None, len(outs) - 1)]
    errs = []
    for W, n, k, src, i in checks:
        xin = h0 if src is None else stack_input(torch, outs[src])
        nl = n // world
        r0 = n * rank // world
        errs.append(oracle_rows_check(torch, W, weight_bytes(DTYPE, 1, k), xin, outs[i][r0:r0 + nl], nl))
    err = torch.tensor([max(errs)], device=dev)
    if world > 1:
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
    e = float(err.item())
    return {"checker": "C oracle (pinned bit for bit to the reference build)", "tol": 1e-3,
            "tasks": "q0, o0, last down, LM head; 16 sampled rows of every rank's slice",
            "max_l2_rel": float(f"{e:.3e}"), "pass": e <= 1e-3}


def check_against_per_gemv(torch, pairs, out, what):
    """The stack against the same GEMVs launched one by one: bit for bit where
    the task reads the stack input (the LM head), and within 1e-4 L2-relative
    where it reads another task's output (the stack hands a dependent task its
    source's output with the lowest mantissa bit cleared, the per-GEMV path the
    exact floats; a 2^-23 change can flip the rounding of a few 16-bit x values
    along a chain of GEMVs).  Parity proper is the oracle check (1e-3)."""
    for name, y in pairs:
        ref = out[name]
        if name == "head":
            ok = torch.equal(y, ref)
        else:
            ok = float(torch.linalg.vector_norm(y - ref) / torch.linalg.vector_norm(ref)) <= 1e-4
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
    out = {}
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
        out[f"M{M}"] = {"ms": round(ms, 3), "tok_s": round(M * 1e3 / ms, 1),
                        "path": "tcgen05" if M >= 16 else "batch-1 kernel per token, per-GEMV launches"}
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
        out["M4_stack"] = {"ms": round(ms, 3), "tok_s": round(M * 1e3 / ms, 1),
                           "path": "GEMV stack once per token"}
        del g
    for M in (2, 3, 4, 8, 16, 64):
        out[f"M{M}_tokens_stack"] = tokens_stack(torch, L, layers, head, M, stream, dev, timed, args, peak)
    return out


def tokens_stack(torch, L, layers, head, M, stream, dev, timed, args, peak):
    """configs[3] at M = 2..4, 8 and 16..64 tokens: the headline's task list
    (same weights, same dependencies) as ONE stack per step
    (nexus_gpu_stack_create_tokens: CUDA cores below 16 tokens, tcgen05 tensor
    cores from 16): every weight read once for all M tokens (M = 8: two
    4-token stacks, each weight read twice).
    Parity: 16 sampled rows of the first q, the first o, the last down and the
    LM head of the first and the last token against the C oracle, each fed the
    input the stack gave it."""
    import ctypes

    from nexusllm_b200 import _native
    from nexusllm_b200.formats import weight_bytes

    tasks, ys = [], []
    inputs_of = {"q": -1, "k": -1, "v": -1, "o": 0, "gate": 3, "up": 3, "down": 4}
    last_down = -1
    for mats in layers:
        base = len(tasks)
        for name, n, k in LAYER_SHAPES:
            y = torch.empty(M, n, dtype=torch.float32, device=dev)
            src = inputs_of[name]
            tasks.append(_native.StackTask(mats[name].data_ptr(), n, k, y.data_ptr(), src if src < 0 else base + src,
                                           last_down if src < 0 else -1))
            ys.append(y)
        last_down = base + 6
    y = torch.empty(M, VOCAB, dtype=torch.float32, device=dev)
    tasks.append(_native.StackTask(head.data_ptr(), VOCAB, HIDDEN, y.data_ptr(), -1, last_down))
    ys.append(y)
    arr = (_native.StackTask * len(tasks))(*tasks)
    h = ctypes.c_void_p()
    _native_check(L.nexus_gpu_stack_create_tokens(DTYPE, arr, len(tasks), HIDDEN, M, ctypes.byref(h)))
    x = torch.randn(M, HIDDEN, generator=torch.Generator(device=dev).manual_seed(60 + M), device=dev)
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            _native_check(L.nexus_gpu_stack_run(h, x.data_ptr(), stream.cuda_stream))
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(g, stream=stream):
                _native_check(L.nexus_gpu_stack_run(h, x.data_ptr(), stream.cuda_stream))
            for _ in range(3):
                g.replay()
        reps = max(5, min(50, args.steps // 20))
        ms = timed(g.replay, reps) / reps
        check_status(L)
        errs = []
        per, nl = 7, len(layers)
        for t in (0, M - 1):
            for W, n, k, src, i in [(layers[0]["q"], HIDDEN, HIDDEN, None, 0), (layers[0]["o"], HIDDEN, HIDDEN, 0, 3),
                                    (layers[-1]["down"], HIDDEN, FFN, per * (nl - 1) + 4, per * (nl - 1) + 6),
                                    (head, VOCAB, HIDDEN, None, len(ys) - 1)]:
                xin = x[t] if src is None else stack_input(torch, ys[src][t])
                errs.append(oracle_rows_check(torch, W, weight_bytes(DTYPE, 1, k), xin, ys[i][t], n))
        del g
    finally:
        L.nexus_gpu_stack_destroy(h)
    sb = step_bytes(layers=len(layers))
    gbs = sb / (ms * 1e-3) / 1e9
    e = max(errs)
    path = ("tcgen05 GEMV stack (persistent, grid barriers at hops), one launch per step" if M >= 16
            else "multi-token CUDA-core GEMV stack, one launch per step" if M <= 4
            else f"{-(-M // 4)} multi-token CUDA-core GEMV stacks of 2-4 tokens per step (weights read {-(-M // 4)}x)")
    return {"ms": round(ms, 3), "tok_s": round(M * 1e3 / ms, 1), "GBs_weights_once": round(gbs, 1),
            "frac": round(gbs / peak, 4), "path": path,
            "parity_max_l2_rel": float(f"{e:.3e}"), "parity_pass": e <= 1e-3}


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
    out = {"cols": "[us per call, % of measured HBM]; rows x cols"}
    for dt, name in ((7, "q4_0"), (9, "q8_0"), (11, "q5_k"), (12, "q6_k"), (1, "fp16")):
        out[name] = {}
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
            out[name][f"{rows}x{cols}"] = [round(ms * 1e3, 2), round(100 * gbs / peak, 1)]
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
    out = {"cols": "[us per call, % of measured HBM]; rows x cols; INT4 group 128 with zeros"}
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
            out.setdefault(fmt, {})[f"{rows}x{cols}"] = [round(ms * 1e3, 2), round(100 * gbs / peak, 1)]
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
    return {"ms_per_step": round(ms, 4), "tokens_per_s": round(1e3 / ms, 2), "GBs": round(gbs, 1),
            "pct_of_measured_hbm": round(100 * gbs / peak, 2),
            "dataflow": "RMSNorm->qkv; o+res; RMSNorm->gate+up pair (SwiGLU); down+res; RMSNorm->head"}


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
            import warnings

            with warnings.catch_warnings():  # read-only memmap views: torch only reads them here
                warnings.simplefilter("ignore", UserWarning)
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
    del write_s
    return {"tensor_bytes": data_bytes, "upload_s": round(best, 4), "upload_gbs": round(gbs, 2),
            "pinned_h2d_gbs": round(pinned_gbs, 2), "frac_of_pinned_h2d": round(gbs / pinned_gbs, 3),
            "plain_per_tensor_pageable_gbs": round(data_bytes / plain_s / 1e9, 2),
            "decode_from_file_ms": round(dec_ms, 4), "load_s": round(load_s, 3)}


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
STACK_TRAFFIC_PER_ALG_BYTE = (786441728 + 4922368) / 788075520  # 4 layers + LM head: read + written / algorithmic


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


# --------------------------------------------------- BASELINE configs[0..2], [4]
def _cpu_time(fn, min_seconds=1.5, min_reps=3):
    """Median seconds of fn() after one warm-up call, over >= min_reps calls and >= min_seconds."""
    fn()
    t, start = [], time.perf_counter()
    while len(t) < min_reps or time.perf_counter() - start < min_seconds:
        t0 = time.perf_counter()
        fn()
        t.append(time.perf_counter() - t0)
    return statistics.median(t), len(t)


def _cpu_legs(mats, alg_bytes, what):
    """NexusLLM's own GEMV over `mats` [(dtype, W, x, y, rows, cols)] on 1 host
    thread and on all host threads: {"1t": ..., "all": ...} with GB/s of
    alg_bytes per pass and ms per pass."""
    import oracle

    if oracle.reference_available():
        lib, kind = oracle.reference(), "reference"
    else:
        lib, kind = oracle.port(), "port"
    out = {"kind": kind}
    del what
    for label, threads in (("1t", 1), ("all", cpu_threads())):
        def one():
            for dt, W, x, y, n, k in mats:
                if kind == "reference":
                    oracle.gemv_threaded(lib, dt, W, x, y, n, k, threads)
                else:
                    y[:] = lib.gemv(dt, W, x, n, k)
        sec, reps = _cpu_time(one)
        out[label] = {"GBs": round(alg_bytes / sec / 1e9, 3), "ms": round(sec * 1e3, 3), "thr": threads}
    return out


def _gpu_gemv_rate(torch, L, dev, timed, dt, rows, cols, seed, min_bytes=512 << 20):
    """Batch-1 GEMVs through nexus_gpu_gemv (x quantization + fused GEMV, two
    launches a call), cycling over enough weight copies (>= min_bytes, far
    beyond the 126 MB L2) that weights come from HBM; a CUDA graph of two
    passes.  Returns (us per call, copies)."""
    from nexusllm_b200 import synth
    from nexusllm_b200.formats import weight_bytes

    wb = weight_bytes(dt, rows, cols)
    n = max(1, -(-min_bytes // wb))
    Ws = [synth.blocks_torch(dt, rows, cols, seed + i, device=dev) for i in range(n)]
    x = torch.randn(cols, device=dev, generator=torch.Generator(device=dev).manual_seed(cols))
    y = torch.empty(rows, device=dev)
    calls = 2 * n

    def run():
        st = torch.cuda.current_stream(dev).cuda_stream
        for i in range(calls):
            rc = L.nexus_gpu_gemv(Ws[i % n].data_ptr(), dt, x.data_ptr(), 0, y.data_ptr(), 1, rows, cols, st)
            if rc:
                raise RuntimeError(L.nexus_gpu_last_error())

    stream = torch.cuda.Stream(dev)
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
    del g, Ws
    return ms * 1e3, n


def make_stack(torch, L, layers, head, m, dt, dev):
    """An unsharded stack of the decode step's GEMVs (same task order and
    dependencies as the headline; head may be None)."""
    import ctypes

    from nexusllm_b200 import _native

    tasks, ys = [], []
    inputs_of = {"q": -1, "k": -1, "v": -1, "o": 0, "gate": 3, "up": 3, "down": 4}
    last_down = -1
    for mats in layers:
        base = len(tasks)
        for name, n, k in shapes_of(m):
            y = torch.empty(n, dtype=torch.float32, device=dev)
            src = inputs_of[name]
            tasks.append(_native.StackTask(mats[name].data_ptr(), n, k, y.data_ptr(),
                                           src if src < 0 else base + src, last_down if src < 0 else -1))
            ys.append(y)
        last_down = base + 6
    if head is not None:
        y = torch.empty(m["vocab"], dtype=torch.float32, device=dev)
        tasks.append(_native.StackTask(head.data_ptr(), m["vocab"], m["hidden"], y.data_ptr(), -1, last_down))
        ys.append(y)
    arr = (_native.StackTask * len(tasks))(*tasks)
    h = ctypes.c_void_p()
    _native.check(L.nexus_gpu_stack_create(dt, arr, len(tasks), m["hidden"], ctypes.byref(h)))
    return h, ys


def _time_stack(torch, L, h, x, dev, timed, reps):
    from nexusllm_b200 import _native

    stream = torch.cuda.Stream(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        _native.check(L.nexus_gpu_stack_run(h, x.data_ptr(), stream.cuda_stream))
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g, stream=stream):
            _native.check(L.nexus_gpu_stack_run(h, x.data_ptr(), stream.cuda_stream))
        for _ in range(3):
            g.replay()
    ms = timed(g.replay, reps) / reps
    check_status(L)
    del g
    return ms


def config0(torch, L, dev, timed, peak):
    """GGUF Q4_0 GEMV, N = K = 4096, batch 1."""
    import numpy as np

    from nexusllm_b200 import synth

    N = K = 4096
    alg = q4_bytes(N, K) + 4 * K + 4 * N
    us, copies = _gpu_gemv_rate(torch, L, dev, timed, DTYPE, N, K, 10_000, min_bytes=600 << 20)
    gbs = alg / (us * 1e-6) / 1e9
    # the same GEMVs as independent tasks of one stack launch (one x, no dependencies)
    import ctypes

    from nexusllm_b200 import _native

    n = 64
    Ws = [synth.blocks_torch(DTYPE, N, K, 10_000 + i, device=dev) for i in range(n)]
    ys = [torch.empty(N, device=dev) for _ in range(n)]
    arr = (_native.StackTask * n)(*[_native.StackTask(W.data_ptr(), N, K, y.data_ptr(), -1, -1)
                                    for W, y in zip(Ws, ys)])
    h = ctypes.c_void_p()
    _native.check(L.nexus_gpu_stack_create(DTYPE, arr, n, K, ctypes.byref(h)))
    x = torch.randn(K, device=dev, generator=torch.Generator(device=dev).manual_seed(K))
    ms = _time_stack(torch, L, h, x, dev, timed, 20)
    L.nexus_gpu_stack_destroy(h)
    del Ws, ys
    sus = ms * 1e3 / n
    sgbs = alg / (sus * 1e-6) / 1e9
    W0 = synth.blocks_numpy(DTYPE, N, K, 10_000)
    xh = synth.activations_numpy(1, K, 10_001)[0]
    mats = [(DTYPE, np.copy(W0), xh, np.zeros(N, np.float32), N, K) for _ in range(64)]
    cpu = _cpu_legs(mats, alg * 64, "64 distinct copies of the 4096x4096 matrix (604 MB) per pass")
    for leg in ("1t", "all"):
        cpu[leg]["ms"] = round(cpu[leg]["ms"] / 64, 4)  # per call
    del copies
    return {"bytes": alg, "gpu": {"us": round(us, 2), "GBs": round(gbs, 1), "frac": round(gbs / peak, 4),
                                  "calls_s": round(1e6 / us)},
            "gpu_stack64": {"us": round(sus, 2), "GBs": round(sgbs, 1), "frac": round(sgbs / peak, 4)},
            "cpu": cpu}


def config1(torch, L, dev, timed, peak):
    """GGUF Q8_0, the Llama-2-7B decode shape set at batch 1: per
    shape, the set (q/k/v/o 4096^2, gate/up 11008x4096, down 4096x11008), and
    the 32-layer stack of those shapes in one launch."""
    import numpy as np

    from nexusllm_b200 import synth
    from nexusllm_b200.formats import weight_bytes

    dt = 9
    m = {"name": "7b", "hidden": 4096, "kv": 4096, "ffn": 11008, "vocab": 32000, "layers": 32}
    per = {}
    for rows, cols in ((4096, 4096), (11008, 4096), (4096, 11008)):
        us, copies = _gpu_gemv_rate(torch, L, dev, timed, dt, rows, cols, 20_000 + rows + cols)
        alg = weight_bytes(dt, rows, cols) + 4 * rows + 4 * cols
        gbs = alg / (us * 1e-6) / 1e9
        per[f"{rows}x{cols}"] = {"us": round(us, 2), "GBs": round(gbs, 1), "frac": round(gbs / peak, 4)}
    set_bytes = sum(weight_bytes(dt, n, k) + 4 * n + 4 * k for _, n, k in shapes_of(m))
    set_us = sum(per[f"{n}x{k}"]["us"] for _, n, k in shapes_of(m))
    layers, _ = gen_model(torch, m, 0, 1, dev, 21_000, dt=dt)
    h, _ys = make_stack(torch, L, layers, None, m, dt, dev)
    x = torch.randn(m["hidden"], device=dev, generator=torch.Generator(device=dev).manual_seed(7))
    ms = _time_stack(torch, L, h, x, dev, timed, 50)
    L.nexus_gpu_stack_destroy(h)
    del layers
    sb = set_bytes * m["layers"]
    sgbs = sb / (ms * 1e-3) / 1e9
    base = [synth.blocks_numpy(dt, n, k, 22_000 + i) for i, (_, n, k) in enumerate(shapes_of(m))]
    xs = {k: synth.activations_numpy(1, k, 22_100 + k)[0] for k in (4096, 11008)}
    mats = [(dt, np.copy(W), xs[k], np.zeros(n, np.float32), n, k)
            for _ in range(3) for W, (_, n, k) in zip(base, shapes_of(m))]
    cpu = _cpu_legs(mats, set_bytes * 3, "3 distinct copies of the 7-GEMV set (645 MB) per pass")
    for leg in ("1t", "all"):
        cpu[leg]["ms"] = round(cpu[leg]["ms"] / 3, 3)  # per 7-GEMV set
    return {"per_shape": per,
            "set": {"us": round(set_us, 2), "GBs": round(set_bytes / (set_us * 1e-6) / 1e9, 1),
                    "frac": round(set_bytes / (set_us * 1e-6) / 1e9 / peak, 4)},
            "stack32": {"ms": round(ms, 4), "GBs": round(sgbs, 1), "frac": round(sgbs / peak, 4)},
            "cpu": cpu}


def config2(torch, L, dev, timed, peak):
    """GGUF Q5_K and Q6_K over a full 32-layer Llama-2-7B weight
    stack (hidden 4096, FFN 11008; the Q6_K down rows at K = 11008 are 9030 B,
    not 16-byte multiples), batch 1, one stack launch per token."""
    import numpy as np

    from nexusllm_b200 import synth
    from nexusllm_b200.formats import weight_bytes

    m = {"name": "7b", "hidden": 4096, "kv": 4096, "ffn": 11008, "vocab": 32000, "layers": 32}
    out = {}
    for dt, name in ((11, "q5_k"), (12, "q6_k")):
        layers, _ = gen_model(torch, m, 0, 1, dev, 30_000 + 1000 * dt, dt=dt)
        h, _ys = make_stack(torch, L, layers, None, m, dt, dev)
        x = torch.randn(m["hidden"], device=dev, generator=torch.Generator(device=dev).manual_seed(dt))
        ms = _time_stack(torch, L, h, x, dev, timed, 50)
        L.nexus_gpu_stack_destroy(h)
        del layers
        layer_bytes = sum(weight_bytes(dt, n, k) + 4 * n + 4 * k for _, n, k in shapes_of(m))
        sb = layer_bytes * m["layers"]
        gbs = sb / (ms * 1e-3) / 1e9
        base = [synth.blocks_numpy(dt, n, k, 31_000 + i) for i, (_, n, k) in enumerate(shapes_of(m))]
        xs = {k: synth.activations_numpy(1, k, 31_100 + k)[0] for k in (4096, 11008)}
        mats = [(dt, np.copy(W), xs[k], np.zeros(n, np.float32), n, k)
                for _ in range(3) for W, (_, n, k) in zip(base, shapes_of(m))]
        cpu = _cpu_legs(mats, layer_bytes * 3, "3 distinct copies of one layer's 7 GEMVs per pass; ms_per_token = "
                                               "32 x ms_per_layer")
        for leg in ("1t", "all"):
            cpu[leg]["ms"] = round(32 * cpu[leg]["ms"] / 3, 2)  # per token: 32 x one layer
        out[name] = {"gpu": {"ms": round(ms, 4), "GBs": round(gbs, 1), "frac": round(gbs / peak, 4)}, "cpu": cpu}
    return out


def oracle_rows_check(torch, W_slice, row_bytes, xin, got, rows_local, n_sample=16):
    """Sampled rows of this rank's slice of a GEMV against the C oracle (the
    checker, pinned to the reference build): rows spread over the slice, the
    task's own input xin (fp32, as the stack consumed it).  Returns the
    L2-relative error over the sampled rows."""
    import numpy as np

    import oracle

    port = oracle.port()
    idx = np.unique(np.linspace(0, rows_local - 1, n_sample).astype(np.int64))
    wb = W_slice.view(-1)
    Wh = np.concatenate([wb[int(r) * row_bytes:(int(r) + 1) * row_bytes].cpu().numpy() for r in idx])
    want = port.gemv(DTYPE, Wh, xin.cpu().numpy().astype(np.float32), len(idx), xin.numel())
    return oracle.l2_rel(got[torch.as_tensor(idx, device=got.device)].cpu().numpy(), want)


def stack_input(torch, y):
    """A task's output as a dependent task of the stack consumes it (the lowest
    mantissa bit, which carries the run's parity, cleared)."""
    return (y.view(torch.int32) & ~1).view(torch.float32)


def model_70b(torch, L, world, rank, local, dev, timed, peak, args, pg):
    """Llama-3-70B Q4_0 (hidden 8192, GQA k/v 1024 x 8192,
    FFN 28672, 80 layers, LM head 128256 x 8192; 39.1 GB per token), row-sharded
    over this run's N GPUs, the same model at every N (seeded by global row).
      m1:  batch 1 -- ONE (sharded) GEMV-stack launch per token; at N > 1 every
           output row goes to every rank by peer stores inside the kernel.
      m16: batch 16 -- 561 GEMVs with 16 activation rows each on the tcgen05
           tensor cores, each rank its row slice, the output slices all-gathered
           with NCCL (N > 1) and re-laid out for the next GEMV; CUDA graph.
      parity: sampled rows of every rank's slice of four tasks against the C
           oracle, each with the input the stack gave it (max over ranks)."""
    import ctypes

    import torch.distributed as dist

    from nexusllm_b200 import _native
    from nexusllm_b200.formats import weight_bytes

    m = model_dims("70b")
    layers, head = gen_model(torch, m, rank, world, dev, 7000)
    h0 = torch.randn(m["hidden"], generator=torch.Generator(device=dev).manual_seed(70), device=dev)
    sb = model_bytes(m)
    tasks = []
    inputs_of = {"q": -1, "k": -1, "v": -1, "o": 0, "gate": 3, "up": 3, "down": 4}
    last_down = -1
    names = []
    for mats in layers:
        base = len(tasks)
        for name, n, k in shapes_of(m):
            src = inputs_of[name]
            tasks.append((mats[name], n, k, src if src < 0 else base + src, last_down if src < 0 else -1))
            names.append(name)
        last_down = base + 6
    tasks.append((head, m["vocab"], m["hidden"], -1, last_down))
    names.append("head")
    # ---- m1: the stack
    if world == 1:
        h, outs = make_stack(torch, L, layers, head, m, DTYPE, dev)
        st_obj = None
    else:
        from nexusllm_b200.sharded import ShardedStack

        st_obj = ShardedStack(DTYPE, [(W.data_ptr(), n, k, src, after) for W, n, k, src, after in tasks],
                              m["hidden"], world, rank)
        h = st_obj.handle
        outs = [torch.as_tensor(_DeviceVec(st_obj.output(i), n), device=dev) for i, (_, n, *_r) in enumerate(tasks)]
    stream = torch.cuda.Stream(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        _native.check(L.nexus_gpu_stack_run(h, h0.data_ptr(), stream.cuda_stream))
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier(device_ids=[local])
        with torch.cuda.graph(g, stream=stream):
            _native.check(L.nexus_gpu_stack_run(h, h0.data_ptr(), stream.cuda_stream))
        for _ in range(max(3, args.warmup)):
            g.replay()
    reps = max(5, min(args.steps, 50))
    ms1 = timed(g.replay, reps) / reps
    check_status(L)
    # parity of sampled rows (this rank's slice), each task with its own input as the stack consumed it
    rb = weight_bytes(DTYPE, 1, m["hidden"])
    errs = []
    for i in (0, 3, len(tasks) - 2, len(tasks) - 1):  # q and o of layer 0, the last down, the LM head
        W, n, k, src, _ = tasks[i]
        r0 = n * rank // world
        xin = h0 if src < 0 else stack_input(torch, outs[src])
        nl = n // world
        errs.append(oracle_rows_check(torch, W, weight_bytes(DTYPE, 1, k), xin, outs[i][r0:r0 + nl], nl))
    err = torch.tensor([max(errs)], device=dev)
    if world > 1:
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
    err = float(err.item())
    del g
    if world > 1:
        dist.barrier(device_ids=[local])
    if st_obj is not None:
        st_obj.close()
    else:
        L.nexus_gpu_stack_destroy(h)
    gbs1 = sb / (ms1 * 1e-3) / 1e9
    out = {"n_gpus": world,
           "m1": {"ms": round(ms1, 4), "tok_s": round(1e3 / ms1, 2), "agg_GBs": round(gbs1, 1),
                  "frac_per_gpu": round(gbs1 / world / peak, 4)},
           "parity": {"max_l2_rel": float(f"{err:.3e}"), "pass": err <= 1e-3}}
    # ---- m16: batched, per-GEMV tensor-core launches (+ NCCL all-gathers)
    M = 16
    ws_need = max([L.nexus_gpu_gemv_workspace_size(DTYPE, M, n // world, k) for _, n, k in shapes_of(m)] +
                  [L.nexus_gpu_gemv_workspace_size(DTYPE, M, m["vocab"] // world, m["hidden"])])
    ws = torch.empty(ws_need + 256, dtype=torch.uint8, device=dev)
    X0 = torch.randn(M, m["hidden"], device=dev, generator=torch.Generator(device=dev).manual_seed(16))
    rows_of = {"q": m["hidden"], "k": m["kv"], "v": m["kv"], "o": m["hidden"], "gate": m["ffn"], "up": m["ffn"],
               "down": m["hidden"], "head": m["vocab"]}
    part = {key: torch.empty(M, n // world, device=dev) for key, n in rows_of.items()}
    gath = {key: torch.empty(world, M, n // world, device=dev) for key, n in rows_of.items()} if world > 1 else None
    full = {key: torch.empty(M, n, device=dev) for key, n in rows_of.items()} if world > 1 else part

    def gemv16(W, n, k, X, key):
        st = torch.cuda.current_stream(dev).cuda_stream
        rc = L.nexus_gpu_gemv_ws(W.data_ptr(), DTYPE, X.data_ptr(), 0, part[key].data_ptr(), M, n // world, k,
                                 ws.data_ptr(), ws.numel(), st)
        if rc:
            raise RuntimeError(L.nexus_gpu_last_error())
        if world > 1:  # every rank's [M, n/world] slice -> the full [M, n] rows of the next GEMV's x
            dist.all_gather_into_tensor(gath[key], part[key], group=pg)
            full[key].copy_(gath[key].permute(1, 0, 2).reshape(M, n))
        return full[key]

    def step16():
        for mats in layers:
            q = gemv16(mats["q"], m["hidden"], m["hidden"], X0, "q")
            gemv16(mats["k"], m["kv"], m["hidden"], X0, "k")
            gemv16(mats["v"], m["kv"], m["hidden"], X0, "v")
            o = gemv16(mats["o"], m["hidden"], m["hidden"], q, "o")
            gt = gemv16(mats["gate"], m["ffn"], m["hidden"], o, "gate")
            gemv16(mats["up"], m["ffn"], m["hidden"], o, "up")
            gemv16(mats["down"], m["hidden"], m["ffn"], gt, "down")
        gemv16(head, m["vocab"], m["hidden"], X0, "head")

    with torch.cuda.stream(stream):
        step16()
    torch.cuda.synchronize(dev)
    g16 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g16, stream=stream):
        step16()
    with torch.cuda.stream(stream):
        for _ in range(3):
            g16.replay()
    reps16 = max(3, min(args.steps, 20))
    ms16 = timed(g16.replay, reps16) / reps16
    del g16
    gbs16 = (sum(weight_bytes(DTYPE, n, k) for _, n, k in shapes_of(m)) * m["layers"] +
             weight_bytes(DTYPE, m["vocab"], m["hidden"])) / (ms16 * 1e-3) / 1e9
    out["m16"] = {"ms": round(ms16, 4), "tok_s": round(M * 1e3 / ms16, 1), "agg_weight_GBs": round(gbs16, 1),
                  "path": "tcgen05 per GEMV" + (" + NCCL all-gathers" if world > 1 else "")}
    if world == 1:
        # ---- m16 as one tensor-core stack launch per step (the same GEMVs and inputs)
        import ctypes

        from nexusllm_b200 import _native

        tasks, ys = [], []
        src_of = {"q": -1, "k": -1, "v": -1, "o": 0, "gate": 3, "up": 3, "down": 4}
        for mats in layers:
            b0 = len(tasks)
            for name, n, k in shapes_of(m):
                y = torch.empty(M, n, device=dev)
                ys.append(y)
                src = src_of[name]
                tasks.append(_native.StackTask(mats[name].data_ptr(), n, k, y.data_ptr(), src if src < 0 else b0 + src,
                                               -1))
        y = torch.empty(M, m["vocab"], device=dev)
        ys.append(y)
        tasks.append(_native.StackTask(head.data_ptr(), m["vocab"], m["hidden"], y.data_ptr(), -1, -1))
        arr = (_native.StackTask * len(tasks))(*tasks)
        hs = ctypes.c_void_p()
        _native_check(L.nexus_gpu_stack_create_tokens(DTYPE, arr, len(tasks), m["hidden"], M, ctypes.byref(hs)))
        try:
            gs = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                _native_check(L.nexus_gpu_stack_run(hs, X0.data_ptr(), stream.cuda_stream))
                torch.cuda.synchronize(dev)
                with torch.cuda.graph(gs, stream=stream):
                    _native_check(L.nexus_gpu_stack_run(hs, X0.data_ptr(), stream.cuda_stream))
                for _ in range(3):
                    gs.replay()
            mss = timed(gs.replay, reps16) / reps16
            check_status(L)
            # the LM head of the stack equals the per-GEMV path's (same input, same arithmetic)
            err16 = float(torch.linalg.vector_norm(ys[-1] - full["head"]) / torch.linalg.vector_norm(full["head"]))
            del gs
        finally:
            L.nexus_gpu_stack_destroy(hs)
        gbss = gbs16 * ms16 / mss
        out["m16_stack"] = {"ms": round(mss, 4), "tok_s": round(M * 1e3 / mss, 1), "agg_weight_GBs": round(gbss, 1),
                            "path": "tcgen05 GEMV stack, one launch per step",
                            "head_vs_per_gemv_l2_rel": float(f"{err16:.3e}")}
        del ys
    del layers, head, ws, full, part, gath
    torch.cuda.empty_cache()
    return out


if __name__ == "__main__":
    main()
