"""GgufDecodeStack's checks that run before any device is touched: one stack
format for every matrix, fp32 norms of the hidden size."""
import numpy as np
import pytest

from nexusllm_b200 import gguf
from nexusllm_b200.decode import GgufDecodeStack


def _write(path, q_type=gguf.GGML_Q4_0, norm_len=256, H=256):
    blocks = {gguf.GGML_Q4_0: 18, gguf.GGML_Q8_0: 34}
    t = []
    for name, rows, cols in [("attn_q", H, H), ("attn_k", 64, H), ("attn_v", 64, H), ("attn_output", H, H),
                             ("ffn_gate", 512, H), ("ffn_up", 512, H), ("ffn_down", H, 512)]:
        gt = q_type if name == "attn_q" else gguf.GGML_Q4_0
        if gt == gguf.GGML_F16:
            data = np.zeros(rows * cols, np.float16).tobytes()
        else:
            data = bytes(rows * cols // 32 * blocks[gt])
        t.append((f"blk.0.{name}.weight", gt, [cols, rows], data))
    t += [("blk.0.attn_norm.weight", gguf.GGML_F32, [norm_len], np.ones(norm_len, np.float32).tobytes()),
          ("blk.0.ffn_norm.weight", gguf.GGML_F32, [H], np.ones(H, np.float32).tobytes()),
          ("output_norm.weight", gguf.GGML_F32, [H], np.ones(H, np.float32).tobytes()),
          ("output.weight", gguf.GGML_Q4_0, [H, 100], bytes(100 * H // 32 * 18))]
    gguf.write_gguf(path, [("general.architecture", gguf.STRING, "llama"), ("llama.block_count", gguf.U32, 1)], t)


@pytest.mark.parametrize("kw,msg", [(dict(q_type=gguf.GGML_Q8_0), "one of"), (dict(q_type=gguf.GGML_F16), "one of"),
                                    (dict(norm_len=128), "fp32 weights")])
def test_decode_stack_rejects_unservable_files(tmp_path, kw, msg):
    p = str(tmp_path / "m.gguf")
    _write(p, **kw)
    with pytest.raises(ValueError, match=msg):
        GgufDecodeStack(p)
