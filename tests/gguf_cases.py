"""Synthetic GGUF files for the loader tests (deterministic: the same bytes on
every machine), shared by tests/test_gguf.py, tests/test_gguf_gpu.py and
tests/golden/make_golden.py, which records what NexusLLM's own loader reads
from them into tests/golden/gguf_ref.json."""
from __future__ import annotations

import os
import struct

import numpy as np

from nexusllm_b200 import gguf as G


def _rand(seed: int, n: int) -> bytes:
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8).tobytes()


def _q8_rows(seed: int, rows: int, cols: int) -> bytes:
    """Q8_0 blocks with finite fp16 scales."""
    r = np.random.default_rng(seed)
    nb = rows * cols // 32
    d = (r.uniform(0.001, 0.05, nb).astype(np.float16)).view(np.uint8).reshape(nb, 2)
    q = r.integers(0, 256, (nb, 32), dtype=np.uint8)
    return np.concatenate([d, q], axis=1).tobytes()


def _q4_rows(seed: int, rows: int, cols: int) -> bytes:
    r = np.random.default_rng(seed)
    nb = rows * cols // 32
    d = (r.uniform(0.001, 0.05, nb).astype(np.float16)).view(np.uint8).reshape(nb, 2)
    q = r.integers(0, 256, (nb, 16), dtype=np.uint8)
    return np.concatenate([d, q], axis=1).tobytes()


def reference_fixture(path: str, hidden: int = 64, layers: int = 2, vocab: int = 256, exclude=()):
    """The layout of the reference's own GGUF test file (tests/
    test_gguf_binary_mmap.py:21-162 in NexusLLM): llama metadata, FP32
    embeddings/norms/LM head, Q8_0 attention, Q4_0 FFN, data back to back."""
    ffn = hidden * 2
    md = [("general.architecture", G.STRING, "llama"), ("general.alignment", G.U32, 32),
          ("llama.context_length", G.U32, 512), ("llama.embedding_length", G.U32, hidden),
          ("llama.feed_forward_length", G.U32, ffn), ("llama.block_count", G.U32, layers),
          ("llama.attention.head_count", G.U32, 2), ("llama.attention.head_count_kv", G.U32, 2),
          ("llama.rope.freq_base", G.F32, 10000.0), ("llama.attention.layer_norm_rms_epsilon", G.F32, 1e-5),
          ("tokenizer.ggml.tokens", G.ARRAY, (G.STRING, [f"tok_{i}" for i in range(vocab)]))]
    norm = struct.pack(f"<{hidden}f", *([1.0] * hidden))
    q8 = (struct.pack("<H", 0x3C00) + b"\x01" * 32) * (hidden * hidden // 32)
    q4 = (struct.pack("<H", 0x3C00) + b"\x11" * 16) * (ffn * hidden // 32)
    t = [("token_embd.weight", G.GGML_F32, [hidden, vocab], bytes(vocab * hidden * 4))]
    for l in range(layers):
        p = f"blk.{l}."
        t += [(p + "attn_norm.weight", G.GGML_F32, [hidden], norm),
              (p + "attn_q.weight", G.GGML_Q8_0, [hidden, hidden], q8),
              (p + "attn_k.weight", G.GGML_Q8_0, [hidden, hidden], q8),
              (p + "attn_v.weight", G.GGML_Q8_0, [hidden, hidden], q8),
              (p + "attn_output.weight", G.GGML_Q8_0, [hidden, hidden], q8),
              (p + "ffn_norm.weight", G.GGML_F32, [hidden], norm),
              (p + "ffn_gate.weight", G.GGML_Q4_0, [hidden, ffn], q4),
              (p + "ffn_up.weight", G.GGML_Q4_0, [hidden, ffn], q4),
              (p + "ffn_down.weight", G.GGML_Q4_0, [ffn, hidden], q4)]
    t += [("output_norm.weight", G.GGML_F32, [hidden], norm),
          ("output.weight", G.GGML_F32, [hidden, vocab], bytes(vocab * hidden * 4))]
    t = [x for x in t if x[0] not in exclude]
    G.write_gguf(path, md, t, alignment=32)
    return t


def mixed_types(path: str, nested: bool = False):
    """Every ggml type the loaders know, metadata of every value type (u64,
    f64, bool, arrays of numbers and strings), alignment 64, MoE keys.
    nested: also an array of arrays, which the reference's parser cannot skip
    (it steps over nested elements as single bytes, model_loader.cpp:589-596)."""
    md = [("general.architecture", G.STRING, "qwen2"), ("general.alignment", G.U32, 64),
          ("general.quantized", G.BOOL, True), ("general.count", G.I32, -7),
          ("qwen2.context_length", G.U64, 32768), ("qwen2.embedding_length", G.U16, 512),
          ("qwen2.feed_forward_length", G.U32, 1536), ("qwen2.block_count", G.U8, 3),
          ("qwen2.attention.head_count", G.U32, 8), ("qwen2.attention.head_count_kv", G.U32, 2),
          ("qwen2.rope.freq_base", G.F64, 1000000.0), ("qwen2.attention.layer_norm_rms_epsilon", G.F64, 1e-6),
          ("qwen2.vocab_size", G.U32, 1000), ("qwen2.expert_count", G.U32, 8),
          ("qwen2.expert_used_count", G.U32, 2), ("tokenizer.ggml.scores", G.ARRAY, (G.F32, [0.5] * 10)),
          ("tokenizer.ggml.merges", G.ARRAY, (G.STRING, ["a b", "c d"]))]
    if nested:
        md.insert(2, ("general.flags", G.ARRAY, (G.ARRAY, [(G.U8, [1, 2, 3]), (G.STRING, ["x", "yz"])])))
    t, seed = [], 0
    for name, gtype, dims, n in [("blk.0.attn_q.weight", G.GGML_Q4_0, [512, 64], 64 * 16 * 18),
                                 ("blk.0.attn_k.weight", G.GGML_Q4_1, [512, 16], 16 * 16 * 20),
                                 ("blk.0.attn_v.weight", G.GGML_Q5_0, [512, 16], 16 * 16 * 22),
                                 ("blk.0.attn_output.weight", G.GGML_Q5_1, [512, 8], 8 * 16 * 24),
                                 ("blk.0.ffn_gate.weight", G.GGML_Q8_0, [512, 48], 48 * 16 * 34),
                                 ("blk.0.ffn_up.weight", G.GGML_Q8_1, [512, 8], 8 * 16 * 36),
                                 ("blk.1.attn_q.weight", G.GGML_Q2_K, [512, 4], 4 * 2 * 84),
                                 ("blk.1.attn_k.weight", G.GGML_Q3_K, [512, 4], 4 * 2 * 110),
                                 ("blk.1.attn_v.weight", G.GGML_Q4_K, [512, 4], 4 * 2 * 144),
                                 ("blk.1.attn_output.weight", G.GGML_Q5_K, [512, 40], 40 * 2 * 176),
                                 ("blk.1.ffn_gate.weight", G.GGML_Q6_K, [512, 40], 40 * 2 * 210),
                                 ("blk.1.ffn_up.weight", G.GGML_Q8_K, [512, 4], 4 * 2 * 292),
                                 ("blk.2.attn_norm.weight", G.GGML_F32, [512], 512 * 4),
                                 ("blk.2.attn_q.weight", G.GGML_F16, [512, 24], 24 * 512 * 2),
                                 ("blk.2.attn_k.weight", G.GGML_BF16, [512, 8], 8 * 512 * 2),
                                 ("blk.2.attn_v.weight", G.GGML_I8, [512, 8], 8 * 512),
                                 ("blk.2.ffn_norm.weight", 26, [512], 512 * 4),
                                 ("token_embd.weight", G.GGML_Q8_0, [512, 1000], 1000 * 16 * 34),
                                 ("output.weight", G.GGML_Q6_K, [512, 1000], 1000 * 2 * 210)]:
        seed += 1
        if gtype == G.GGML_Q8_0:
            data = _q8_rows(seed, dims[1], dims[0])
        elif gtype == G.GGML_Q4_0:
            data = _q4_rows(seed, dims[1], dims[0])
        else:
            data = _rand(seed, n)
        assert len(data) == n, name
        t.append((name, gtype, dims, data))
    G.write_gguf(path, md, t, alignment=64)
    return t


def fallbacks(path: str):
    """Zeroed dimensions the loader infers (model_loader.cpp:803-824), HF-style
    names, tied embeddings (no LM head), a tensor starting past the end of the
    file and one running past it."""
    md = [("general.architecture", G.STRING, "mistral"), ("mistral.embedding_length", G.U32, 0),
          ("mistral.block_count", G.U32, 0), ("mistral.attention.head_count", G.U32, 0),
          ("mistral.attention.head_count_kv", G.U32, 0), ("mistral.feed_forward_length", G.U32, 0),
          ("mistral.vocab_size", G.U32, 0), ("mistral.rope.freq_base", G.U32, 500000),
          ("mistral.attention.layer_norm_rms_epsilon", G.U32, 0)]
    t = [("model.embed_tokens.weight", G.GGML_Q8_0, [256, 500], _q8_rows(11, 500, 256)),
         ("model.layers.0.self_attn.q_proj.weight", G.GGML_Q4_0, [256, 256], _q4_rows(12, 256, 256)),
         ("model.layers.0.mlp.gate_proj.weight", G.GGML_Q4_0, [256, 64], _q4_rows(13, 64, 256)),
         ("model.layers.3.mlp.down_proj.weight", G.GGML_Q4_0, [64, 256], _q4_rows(14, 256, 64)),
         ("model.norm.weight", G.GGML_F32, [256], _rand(15, 1024)),
         ("model.layers.1.self_attn.k_proj.weight", G.GGML_Q4_0, [256, 64], _q4_rows(16, 64, 256)),
         ("model.layers.2.self_attn.v_proj.weight", G.GGML_Q4_0, [256, 64], _q4_rows(17, 64, 256))]
    G.write_gguf(path, md, t, alignment=32)
    # point the last two tensors' table offsets past the end / across it
    size = os.path.getsize(path)
    n_other = len(t) - 2
    layout, pos = [], 0
    for _, _, _, data in t:
        pos = (pos + 31) // 32 * 32
        layout.append(pos)
        pos += len(data)
    data_base = size - pos
    offsets = layout[:n_other] + [size - data_base - 4096 + 4096 * 4,   # starts past the end
                                  size - data_base - 100]               # starts inside, runs past the end
    G.write_gguf(path, md, t, alignment=32, offsets=offsets)
    return t


CASES = {"reference_fixture": reference_fixture, "mixed_types": mixed_types, "fallbacks": fallbacks,
         "nested_array": lambda p: mixed_types(p, nested=True)}

# ggml types the reference maps onto another type's DataType (model_loader.cpp:
# 735-746): type -> the reference's DataType; this library reports -1.
REFERENCE_REMAPS = {3: 7, 7: 10, 9: 9, 15: 0, 24: 2, 26: 2}

# names looked up in every case: all tensor names plus canonical aliases
ALIASES = ["token_embd", "token_embd.weight", "lm_head", "output.weight", "output_norm", "model.norm.weight",
           "layers.0.wq", "layers.0.wk", "layers.0.wv", "layers.0.wo", "layers.0.ffn_gate", "layers.0.ffn_up",
           "layers.0.ffn_down", "layers.0.attn_norm", "layers.0.ffn_norm", "layers.1.wq", "layers.1.wk",
           "layers.2.wv", "layers.3.ffn_down", "blk.0.attn_q.weight", "model.layers.0.self_attn.q_proj.weight",
           "layers.9.wq", "no.such.tensor"]


def build(dirpath: str) -> dict:
    """Writes every case under dirpath: {case: (path, tensor list)}."""
    out = {}
    for name, fn in CASES.items():
        p = os.path.join(dirpath, name + ".gguf")
        out[name] = (p, fn(p))
    return out
