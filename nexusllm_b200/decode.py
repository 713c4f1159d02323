"""A decode step on the GPU straight from a GGUF file: the GEMV side of
NexusLLM's ForwardPassExecutor::forward_token (src/forward_pass.cpp:504-585)
with its weights uploaded once and kept in HBM.

`GgufDecodeStack(path)` resolves every layer's tensors through the
reference's names (layers.L.wq, ... -- the loader's alias classes), uploads
the matrices and the RMSNorm weights into one device image
(nexus_gpu_gguf_upload), and builds one fused GEMV stack
(nexus_gpu_stack_create_ex) per token:

    per layer:  RMSNorm -> q, k, v;  o (+ residual);
                RMSNorm -> gate+up pair with the SwiGLU epilogue;  down (+ residual)
    then:       final RMSNorm -> LM head logits

Attention (RoPE, the KV cache, softmax) is not part of this path: the o
projection reads q's output in its place, as the benchmark does.  An engine
with its own attention splits the task list at each attention.
"""
from __future__ import annotations

import ctypes

from . import _native
from .gguf import GGUFFile

_LAYER = ("attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")
_STACK_DTYPES = {7, 9, 11, 12}  # the GGUF formats GEMV stacks serve (Q4_0, Q8_0, Q5_K, Q6_K)


class GgufDecodeStack:
    def __init__(self, path: str, device: str = "cuda", layers: int | None = None):
        import torch

        self.L = _native.lib()
        with GGUFFile(path) as f:
            m = f.model
            n_layers = m["num_hidden_layers"] if layers is None else layers
            names = [f"layers.{l}.{t}" for l in range(n_layers) for t in _LAYER] + ["output_norm", "lm_head"]
            info = {n: f.tensors[f.find(n)] for n in names}
            mats = [n for n in names if not n.endswith("norm")]
            dtypes = {info[n]["dtype"] for n in mats}
            if len(dtypes) != 1 or not dtypes <= _STACK_DTYPES:
                raise ValueError(f"the stack needs one of Q4_0/Q8_0/Q5_K/Q6_K for every matrix, got {dtypes}")
            hidden = info["layers.0.wq"]["cols"]
            for n in names:
                if n.endswith("norm") and (info[n]["dtype"] != 0 or info[n]["cols"] != hidden):
                    raise ValueError(f"{n}: expected {hidden} fp32 weights")
            self.image, placed = f.upload(names, device=device)
        self.dtype, self.hidden, self.eps = dtypes.pop(), hidden, float(m["rms_norm_eps"])
        base = self.image.data_ptr()
        ptr = {n: base + placed[n][0] for n in names}
        self.outputs = []   # (task name, device fp32 output)
        tasks = []
        prev = -1           # the residual stream: the stack input for layer 0

        def task(name, rows, cols, src, res=-2, norm=None, w_up=None):
            y = torch.empty(rows, dtype=torch.float32, device=device)
            self.outputs.append((name, y))
            tasks.append(_native.StackTaskEx(ptr[name], rows, cols, y.data_ptr(), src, -1, -1, res,
                                             None if norm is None else ptr[norm], self.eps,
                                             None if w_up is None else ptr[w_up]))
            return len(tasks) - 1

        for l in range(n_layers):
            p = f"layers.{l}."
            rows = {t: info[p + t]["rows"] for t in ("wq", "wk", "wv", "wo", "ffn_gate", "ffn_down")}
            q = task(p + "wq", rows["wq"], hidden, prev, norm=p + "attn_norm")
            task(p + "wk", rows["wk"], hidden, prev, norm=p + "attn_norm")
            task(p + "wv", rows["wv"], hidden, prev, norm=p + "attn_norm")
            o = task(p + "wo", rows["wo"], rows["wq"], q, res=prev)
            ff = task(p + "ffn_gate", rows["ffn_gate"], hidden, o, norm=p + "ffn_norm", w_up=p + "ffn_up")
            prev = task(p + "ffn_down", rows["ffn_down"], rows["ffn_gate"], ff, res=o)
        task("lm_head", info["lm_head"]["rows"], hidden, prev, norm="output_norm")
        arr = (_native.StackTaskEx * len(tasks))(*tasks)
        self._h = ctypes.c_void_p()
        _native.check(self.L.nexus_gpu_stack_create_ex(self.dtype, arr, len(tasks), hidden, 1, 0,
                                                       ctypes.byref(self._h)))
        self.tasks = tasks

    def step(self, hidden_state, stream=None):
        """Runs the decode step on a device fp32 [hidden] input (16-byte
        aligned); returns the logits tensor (device, overwritten each step)."""
        import torch

        st = stream.cuda_stream if stream is not None else torch.cuda.current_stream().cuda_stream
        _native.check(self.L.nexus_gpu_stack_run(self._h, hidden_state.data_ptr(), st))
        return self.outputs[-1][1]

    def close(self) -> None:
        if self._h:
            self.L.nexus_gpu_stack_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
