"""GGUF file -> device upload (nexus_gpu_gguf_upload) on the GPU: every
uploaded tensor's device bytes equal its bytes in the file (bit-exact, padding
zeroed), an upload large enough to wrap the staging ring, and GEMVs straight
from the uploaded image against the C oracle on the file's bytes."""
import ctypes

import numpy as np
import pytest

import gguf_cases
import oracle
from nexusllm_b200 import _native, gguf

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-3


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return gguf_cases.build(str(tmp_path_factory.mktemp("gguf_gpu")))


def _check_image(path, f, image, placed):
    raw = np.fromfile(path, dtype=np.uint8)
    host = image.cpu().numpy()
    ends = []
    for name, (off, t) in placed.items():
        np.testing.assert_array_equal(host[off:off + t["bytes"]], raw[t["file_offset"]:t["file_offset"] + t["bytes"]],
                                      err_msg=name)
        assert off % 256 == 0
        ends.append((off, off + t["bytes"]))
    ends.sort()
    for (_, e), (s, _) in zip(ends, ends[1:]):  # padding between tensors is zero
        assert not host[e:s].any()


@pytest.mark.parametrize("case", ["reference_fixture", "mixed_types", "fallbacks"])
def test_upload_is_bit_exact(files, case):
    path, _ = files[case]
    with gguf.GGUFFile(path) as f:
        names = [t["name"] for t in f.tensors if t["dtype"] >= 0]
        image, placed = f.upload(names)
        torch.cuda.synchronize()
        _check_image(path, f, image, placed)


def test_upload_wraps_the_staging_ring(tmp_path):
    """~300 MB in 64 MiB pieces through a ring of 4 staging buffers, with
    tensor boundaries inside pieces and tensors larger than a piece."""
    rng = np.random.default_rng(5)
    t = []
    for i, rows in enumerate([20000, 7, 80000, 1, 31000, 5]):
        data = rng.integers(0, 256, rows * 4096 // 32 * 18, dtype=np.uint8).tobytes()
        t.append((f"blk.{i}.ffn_up.weight", gguf.GGML_Q4_0, [4096, rows], data))
    path = str(tmp_path / "big.gguf")
    gguf.write_gguf(path, [("general.architecture", gguf.STRING, "llama")], t)
    with gguf.GGUFFile(path) as f:
        names = [x[0] for x in t][::-1]           # image order differs from file order
        image, placed = f.upload(names)
        assert image.numel() > 4 * (64 << 20)
        torch.cuda.synchronize()
        _check_image(path, f, image, placed)
        # a second upload into a new image reuses the ring
        image2, placed2 = f.upload(names[:2])
        torch.cuda.synchronize()
        _check_image(path, f, image2, placed2)


def test_gemv_on_uploaded_weights(files):
    """nexus_gpu_gemv reads the uploaded image in place (Q8_0 and Q4_0 of the
    reference's own fixture and of the HF-named file) and agrees with the
    oracle over the file's bytes."""
    L = _native.lib()
    port = oracle.port()
    for case, names in [("reference_fixture", ["layers.0.wq", "layers.1.ffn_gate", "layers.1.ffn_down"]),
                        ("fallbacks", ["layers.0.wq", "layers.0.ffn_gate", "lm_head"]),
                        ("mixed_types", ["layers.0.wq", "layers.0.ffn_gate", "output.weight"])]:
        path, _ = files[case]
        raw = np.fromfile(path, dtype=np.uint8)
        with gguf.GGUFFile(path) as f:
            image, placed = f.upload(names)
            for n in names:
                off, t = placed[n]
                x = np.random.default_rng(len(n)).standard_normal(t["cols"]).astype(np.float32)
                dx = torch.from_numpy(x).cuda()
                y = torch.full((t["rows"],), float("nan"), device="cuda")
                rc = L.nexus_gpu_gemv(image.data_ptr() + off, t["dtype"], dx.data_ptr(), 0, y.data_ptr(), 1,
                                      t["rows"], t["cols"], torch.cuda.current_stream().cuda_stream)
                assert rc == 0, L.nexus_gpu_last_error()
                W = raw[t["file_offset"]:t["file_offset"] + t["bytes"]].copy()
                if t["dtype"] == 1:
                    W = W.view(np.uint16)
                want = port.gemv(t["dtype"], W, x, t["rows"], t["cols"])
                got = y.cpu().numpy()
                if np.isfinite(want).all():
                    assert oracle.l2_rel(got, want) <= TOL, (case, n)
                else:  # random K-quant bytes can hold Inf/NaN scales: the same rows are non-finite
                    np.testing.assert_array_equal(np.isfinite(got), np.isfinite(want))
    bits = ctypes.c_uint32(0)
    assert L.nexus_gpu_device_status(ctypes.byref(bits)) == 0 and bits.value == 0
