"""A decode step from a GGUF file (nexusllm_b200.decode.GgufDecodeStack): the
weights and norms uploaded once from the file, the layers run as one fused
GEMV stack.  Every task's output against the C oracle fed the GPU's own input
to that task and the file's bytes (oracle GEMV, RMSNorm and SwiGLU are
bit-identical to the reference build), within the 1e-3 GEMV tolerance; the
dataflow of src/forward_pass.cpp:504-585 with attention stood in by q -> o."""
import numpy as np
import pytest

import oracle
from nexusllm_b200 import gguf
from nexusllm_b200.decode import GgufDecodeStack

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-3


def _q4(rows, cols, seed):
    r = np.random.default_rng(seed)
    nb = rows * cols // 32
    d = r.uniform(0.005, 0.02, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return np.concatenate([d, r.integers(0, 256, (nb, 16), dtype=np.uint8)], axis=1).tobytes()


def _write_model(path, H=1024, KV=256, F=2048, V=1000, layers=2):
    r = np.random.default_rng(9)
    norm = lambda: (1.0 + 0.1 * r.standard_normal(H)).astype(np.float32).tobytes()  # noqa: E731
    t, seed = [], 0
    for l in range(layers):
        p = f"blk.{l}."
        for name, rows, cols in [("attn_q", H, H), ("attn_k", KV, H), ("attn_v", KV, H), ("attn_output", H, H),
                                 ("ffn_gate", F, H), ("ffn_up", F, H), ("ffn_down", H, F)]:
            seed += 1
            t.append((p + name + ".weight", gguf.GGML_Q4_0, [cols, rows], _q4(rows, cols, seed)))
        t += [(p + "attn_norm.weight", gguf.GGML_F32, [H], norm()), (p + "ffn_norm.weight", gguf.GGML_F32, [H], norm())]
    t += [("output_norm.weight", gguf.GGML_F32, [H], norm()), ("output.weight", gguf.GGML_Q4_0, [H, V], _q4(V, H, 99))]
    md = [("general.architecture", gguf.STRING, "llama"), ("llama.embedding_length", gguf.U32, H),
          ("llama.block_count", gguf.U32, layers), ("llama.feed_forward_length", gguf.U32, F),
          ("llama.attention.layer_norm_rms_epsilon", gguf.F32, 1e-5)]
    gguf.write_gguf(path, md, t)


def test_decode_step_from_gguf_matches_oracle(tmp_path):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    path = str(tmp_path / "model.gguf")
    _write_model(path)
    port = oracle.port()
    raw = np.fromfile(path, dtype=np.uint8)
    with gguf.GGUFFile(path) as f:
        host = {}
        for name in [f"layers.{l}.{k}" for l in range(2) for k in ("wq", "wk", "wv", "wo", "ffn_gate", "ffn_up",
                                                                     "ffn_down", "attn_norm", "ffn_norm")] + \
                ["output_norm", "lm_head"]:
            t = f.tensors[f.find(name)]
            host[name] = (raw[t["file_offset"]:t["file_offset"] + t["bytes"]].copy(), t["rows"], t["cols"])
        eps = float(f.model["rms_norm_eps"])
    with GgufDecodeStack(path) as dec:
        assert dec.dtype == 7 and dec.hidden == 1024 and len(dec.tasks) == 2 * 6 + 1
        x = torch.from_numpy(np.random.default_rng(3).standard_normal(1024).astype(np.float32)).cuda()
        logits = dec.step(x)
        torch.cuda.synchronize()
        out = {name: y.cpu().numpy() for name, y in dec.outputs}
        xin = x.cpu().numpy()

        def norm(v, name):
            return port.rmsnorm(v, host[name][0].view(np.float32), eps)

        def gemv(name, v):
            W, rows, cols = host[name]
            return port.gemv(7, W, v, rows, cols)

        h = xin
        for l in range(2):
            p = f"layers.{l}."
            xn = norm(h, p + "attn_norm")
            for k in ("wq", "wk", "wv"):
                assert oracle.l2_rel(out[p + k], gemv(p + k, xn)) <= TOL, p + k
            o_want = (gemv(p + "wo", out[p + "wq"]) + h).astype(np.float32)
            assert oracle.l2_rel(out[p + "wo"], o_want) <= TOL, p + "wo"
            xf = norm(out[p + "wo"], p + "ffn_norm")
            ff_want = port.swiglu(gemv(p + "ffn_gate", xf), gemv(p + "ffn_up", xf))
            assert oracle.l2_rel(out[p + "ffn_gate"], ff_want) <= TOL, p + "ffn_gate+up"
            d_want = (gemv(p + "ffn_down", out[p + "ffn_gate"]) + out[p + "wo"]).astype(np.float32)
            assert oracle.l2_rel(out[p + "ffn_down"], d_want) <= TOL, p + "ffn_down"
            h = out[p + "ffn_down"]
        assert oracle.l2_rel(logits.cpu().numpy(), gemv("lm_head", norm(h, "output_norm"))) <= TOL
        # the next token's step reuses the resident weights; outputs repeat bit for bit
        first = logits.clone()
        dec.step(x)
        torch.cuda.synchronize()
        assert torch.equal(first, logits)
