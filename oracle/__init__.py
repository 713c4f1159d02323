"""CPU checkers for the quantized GEMV path -- TEST INFRASTRUCTURE ONLY.

Two libraries, both built by oracle/Makefile:

* ``port``      -- oracle/build/liboracle.so, the C restatement in
                   nexus_oracle.c (bit-identical to the reference build on the
                   golden vectors).
* ``reference`` -- oracle/_ref/libnexus_ref.so, NexusLLM's own
                   src/quantization.cpp compiled unmodified (only present where
                   the reference sources were available at build time).
* ``reference_gguf_load`` -- oracle/_ref/libnexus_ref_gguf.so, NexusLLM's
                   GGUF loader (src/model_loader.cpp + memory_tier.cpp)
                   compiled unmodified behind the ref_gguf.cpp shim.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this package, and only to check or to time the CPU path; the product
library never calls into it.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libnexus_ref.so")
REF_GGUF_SO = os.path.join(HERE, "_ref", "libnexus_ref_gguf.so")

# NexusLLM DataType values (include/nexus_common.hpp:244-260)
_NAMES = {1: "fp16", 7: "q4_0", 9: "q8_0", 11: "q5_k", 12: "q6_k"}
_VP, _SZ = ctypes.c_void_p, ctypes.c_size_t


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_VP)


class _Lib:
    def __init__(self, path: str, prefix_gemv: str, prefix_deq: str, f16: str):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (run `make -C oracle`)")
        self.path = path
        self.lib = ctypes.CDLL(path)
        self._g, self._d = prefix_gemv, prefix_deq
        fn = getattr(self.lib, f16)
        fn.restype = ctypes.c_float
        fn.argtypes = [ctypes.c_uint16]
        self._f16 = fn
        for name in _NAMES.values():
            f = getattr(self.lib, prefix_gemv + name)
            f.restype = None
            f.argtypes = [_VP, _VP, _VP, _SZ, _SZ]

    def fp16_to_fp32(self, h: int) -> float:
        return self._f16(h)

    def gemv(self, dtype: int, W: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
        """y[rows] = W . x with x float32[cols]; W raw blocks (or uint16 halves)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rows, np.float32)
        getattr(self.lib, self._g + _NAMES[int(dtype)])(_ptr(W), _ptr(x), _ptr(y), rows, cols)
        return y

    def gemv_batched(self, dtype: int, W: np.ndarray, X: np.ndarray, rows: int, cols: int) -> np.ndarray:
        """M independent batch-1 GEMVs (the reference has no batched path)."""
        X = np.ascontiguousarray(X, dtype=np.float32).reshape(-1, cols)
        return np.stack([self.gemv(dtype, W, X[m], rows, cols) for m in range(X.shape[0])])

    # ------------------------------------ INT4-AWQ / FP8-E4M3 (the reference's
    # QuantizationKernel::fused_gemv_int4 / fused_gemv_fp8 and dequantizers)
    def _fn(self, name: str, argtypes):
        f = getattr(self.lib, name)
        f.restype = None
        f.argtypes = argtypes
        return f

    def gemv_int4(self, W: np.ndarray, x: np.ndarray, scales: np.ndarray, zeros, rows: int, cols: int,
                  group_size: int) -> np.ndarray:
        """y[rows] = W . x; W uint32 [rows][cols/8] (nibble k of word j = column 8j+k),
        scales/zeros float32 [rows][cols/group_size] (zeros may be None)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rows, np.float32)
        z = None if zeros is None else _ptr(np.ascontiguousarray(zeros, np.float32))
        self._fn(self._g + "int4", [_VP, _VP, _VP, _VP, _VP, _SZ, _SZ, _SZ])(
            _ptr(W), _ptr(x), _ptr(np.ascontiguousarray(scales, np.float32)), z, _ptr(y), rows, cols, group_size)
        return y

    def gemv_fp8(self, W: np.ndarray, x: np.ndarray, rows: int, cols: int, scale: float) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rows, np.float32)
        self._fn(self._g + "fp8", [_VP, _VP, _VP, _SZ, _SZ, ctypes.c_float])(_ptr(W), _ptr(x), _ptr(y), rows, cols,
                                                                             scale)
        return y

    def dequantize_int4_awq(self, packed: np.ndarray, scales: np.ndarray, zeros, count: int,
                            group_size: int) -> np.ndarray:
        out = np.zeros(count, np.float32)
        z = None if zeros is None else _ptr(np.ascontiguousarray(zeros, np.float32))
        self._fn(self._d + "int4_awq", [_VP, _VP, _VP, _VP, _SZ, _SZ])(
            _ptr(packed), _ptr(np.ascontiguousarray(scales, np.float32)), z, _ptr(out), count, group_size)
        return out

    def dequantize_fp8_e4m3(self, data: np.ndarray, count: int, scale: float) -> np.ndarray:
        out = np.zeros(count, np.float32)
        self._fn(self._d + "fp8_e4m3", [_VP, _VP, _SZ, ctypes.c_float])(_ptr(data), _ptr(out), count, scale)
        return out

    # --------------------------- decode-layer ops (TransformerOps::rmsnorm, swiglu)
    def rmsnorm(self, x: np.ndarray, w, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        wp = None if w is None else _ptr(np.ascontiguousarray(w, np.float32))
        name = "oracle_rmsnorm" if self._g.startswith("oracle") else "ref_rmsnorm"
        self._fn(name, [_VP, _VP, _VP, _SZ, ctypes.c_float])(_ptr(x), wp, _ptr(out), x.size, eps)
        return out

    def swiglu(self, g: np.ndarray, u: np.ndarray) -> np.ndarray:
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        out = np.zeros_like(g)
        name = "oracle_swiglu" if self._g.startswith("oracle") else "ref_swiglu"
        self._fn(name, [_VP, _VP, _VP, _SZ])(_ptr(g), _ptr(u), _ptr(out), g.size)
        return out

    def dequantize(self, dtype: int, W: np.ndarray, count: int) -> np.ndarray:
        name = _NAMES[int(dtype)]
        out = np.zeros(count, np.float32)
        if name == "fp16" and self._d == "ref_dequantize_":
            # the reference has no named FP16 dequantizer: element-wise decoder
            return np.array([self.fp16_to_fp32(int(h)) for h in W.reshape(-1)[:count]], np.float32)
        per = 1 if name == "fp16" else (32 if name in ("q4_0", "q8_0") else 256)
        f = getattr(self.lib, self._d + name)
        f.restype = None
        f.argtypes = [_VP, _VP, _SZ]
        f(_ptr(W), _ptr(out), count // per)
        return out


def port() -> _Lib:
    lib = _Lib(PORT_SO, "oracle_gemv_", "oracle_dequantize_", "oracle_fp16_to_fp32")
    return lib


def reference() -> "_Lib":
    lib = _Lib(REF_SO, "ref_fused_gemv_", "ref_dequantize_", "ref_fp16_to_fp32")
    f = lib.lib.ref_fused_gemv_threaded
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_uint, _VP, _VP, _VP, _SZ, _SZ, ctypes.c_int]
    return lib


def reference_available() -> bool:
    return os.path.exists(REF_SO)


def gemv_threaded(lib: _Lib, dtype: int, W, x, y, rows: int, cols: int, threads: int) -> None:
    """The reference's GEMV over `threads` host threads (oracle/ref_driver.cpp)."""
    rc = lib.lib.ref_fused_gemv_threaded(int(dtype), _ptr(W), _ptr(x), _ptr(y), rows, cols, threads)
    if rc != 0:
        raise ValueError(f"ref_fused_gemv_threaded returned {rc}")


def l2_rel(a: np.ndarray, b: np.ndarray) -> float:
    """||a - b||_2 / ||b||_2 in float64 (the parity metric of the north star)."""
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / nb) if nb > 0 else float(np.linalg.norm(a - b))


class _RefGgufModel(ctypes.Structure):
    _fields_ = [("architecture", ctypes.c_char * 64), ("vocab_size", ctypes.c_uint32), ("hidden_size", ctypes.c_uint32),
                ("intermediate_size", ctypes.c_uint32), ("num_hidden_layers", ctypes.c_uint32),
                ("num_attention_heads", ctypes.c_uint32), ("num_key_value_heads", ctypes.c_uint32),
                ("max_position_embeddings", ctypes.c_uint32), ("rms_norm_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float), ("is_moe", ctypes.c_uint32), ("num_experts", ctypes.c_uint32),
                ("num_experts_per_tok", ctypes.c_uint32), ("loaded_tensor_count", ctypes.c_uint64)]


class _RefGgufTensor(ctypes.Structure):
    _fields_ = [("found", ctypes.c_int32), ("dtype", ctypes.c_int32), ("n_dims", ctypes.c_uint32),
                ("dims", ctypes.c_uint64 * 8), ("byte_size", ctypes.c_uint64), ("fnv", ctypes.c_uint64)]


def reference_gguf_available() -> bool:
    return os.path.exists(REF_GGUF_SO)


def reference_gguf_load(path: str, names, hash_bytes):
    """NexusLLM's loader on `path` (oracle/ref_gguf.cpp): (status, metadata
    dict, [per-name dict: found, dtype, dims, byte_size, fnv of hash_bytes[i]
    bytes at the tensor's data pointer])."""
    lib = ctypes.CDLL(REF_GGUF_SO)
    f = lib.ref_gguf_load
    f.restype = ctypes.c_int32
    f.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
    n = len(names)
    c_names = (ctypes.c_char_p * max(1, n))(*[x.encode() for x in names])
    hb = (ctypes.c_uint64 * max(1, n))(*hash_bytes)
    out = (_RefGgufTensor * max(1, n))()
    m = _RefGgufModel()
    st = f(path.encode(), ctypes.byref(m), c_names, hb, n, out)
    model = {k: getattr(m, k) for k, _ in m._fields_}
    model["architecture"] = m.architecture.decode()
    res = [{"found": t.found, "dtype": t.dtype, "dims": list(t.dims)[:t.n_dims], "byte_size": t.byte_size,
            "fnv": t.fnv} for t in out[:n]]
    return st, model, res


def fnv1a(data: bytes) -> int:
    """FNV-1a 64 (the hash ref_gguf.cpp reports)."""
    h = 1469598103934665603
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h
