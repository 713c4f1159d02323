"""The C++ drop-in (nexusllm_b200/csrc/dropin.cpp): NexusLLM's own
QuantizationKernel GGUF entry points and an INexusComputeBackend device,
compiled against the reference's unmodified headers and linked to
libnexus_gpu.so.  CPU checks: the drop-in defines exactly the symbols the
reference's src/quantization.cpp defines for those methods (same mangled C++
signatures, include/quantization.hpp:80-153), the translation unit compiles
against the reference headers, and its backend keeps matmul_vec_dispatch's
W == nullptr no-op and refuses a type it does not serve -- no GPU needed."""
import ctypes
import os
import shutil
import subprocess

import pytest

from nexusllm_b200 import build as nb

REF = os.environ.get("NEXUS_REFERENCE_DIR", "/root/reference")
METHODS = ["fused_gemv_q4_0", "fused_gemv_q8_0", "fused_gemv_fp16", "fused_gemv_q5_k", "fused_gemv_q6_k",
           "dequantize_gguf_q4_0", "dequantize_gguf_q5_k", "dequantize_gguf_q6_k"]
need_ref = pytest.mark.skipif(not os.path.exists(os.path.join(REF, "include", "quantization.hpp")),
                              reason="reference headers not present (the prebuilt drop-in is tested on the GPU box)")


def _defined(path):
    out = subprocess.run(["nm", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def _ours(names):
    return {n for n in names if "QuantizationKernel" in n and any(m in n for m in METHODS)}


@need_ref
def test_dropin_defines_the_reference_symbols(tmp_path):
    obj = tmp_path / "quantization.o"
    subprocess.run(["g++", "-std=c++20", "-O0", "-mavx2", "-mfma", "-c", f"-I{REF}/include",
                    os.path.join(REF, "src", "quantization.cpp"), "-o", str(obj)], check=True)
    want = _ours(_defined(str(obj)))
    assert len(want) == len(METHODS), sorted(want)
    so = tmp_path / "libnexus_dropin.so"
    nb.build_dropin(os.path.join(REF, "include"), out=str(so))
    got = _ours(_defined(str(so)))
    assert got == want


@need_ref
def test_dropin_translation_unit_compiles_against_reference_headers():
    res = subprocess.run([shutil.which("g++") or "g++", "-std=c++20", "-fsyntax-only", "-Wall", "-Wextra",
                          f"-I{REF}/include", nb.DROPIN_SRC], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


@pytest.mark.skipif(not os.path.exists(nb.DROPIN_OUT), reason="drop-in not built (no reference headers at build)")
def test_backend_keeps_the_no_op_and_refuses_unserved_types():
    lib = ctypes.CDLL(nb.DROPIN_OUT)
    fn = lib.nexus_dropin_backend_gemv
    fn.restype = ctypes.c_int32
    fn.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                   ctypes.c_size_t]
    x = (ctypes.c_float * 64)()
    y = (ctypes.c_float * 4)()
    assert fn(None, 7, x, y, 4, 64) == 0          # W == nullptr: no-op (include/transformer_ops.hpp:158)
    w = (ctypes.c_uint8 * 1024)()
    assert fn(w, 0, x, y, 4, 64) == -3            # FP32: not this device's (its fallback's)
    name = ctypes.create_string_buffer(256)
    kind = ctypes.c_uint32(99)
    assert lib.nexus_dropin_backend_name(name, 256, ctypes.byref(kind)) == 0
    assert kind.value == 1                        # ComputeDeviceType::DEVICE_CUDA
