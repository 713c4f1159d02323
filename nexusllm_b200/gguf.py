"""GGUF files on the GEMV path: the on-disk side of NexusLLM's loader
(UniversalModelLoader::load_gguf, src/model_loader.cpp:416-836) feeding the
device-resident weights the GEMV kernels read.

`GGUFFile` wraps the library's parser and uploader (nexus_gpu_gguf_* in
include/nexus_gpu.h): the file's model metadata and tensor table, and
`upload()` of chosen tensors into one device image (a torch uint8 CUDA
tensor) through pinned staging buffers.  `write_gguf` writes a GGUF v3 file
(used for synthetic models in the tests and the benchmark).
"""
from __future__ import annotations

import ctypes
import struct

from . import _native

# ggml tensor type ids (the values stored in GGUF files)
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1 = 0, 1, 2, 3
GGML_Q5_0, GGML_Q5_1, GGML_Q8_0, GGML_Q8_1 = 6, 7, 8, 9
GGML_Q2_K, GGML_Q3_K, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_K = 10, 11, 12, 13, 14, 15
GGML_I8, GGML_BF16 = 24, 30

# GGUF metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
           U64: "<Q", I64: "<q", F64: "<d"}


def _value(vtype, v) -> bytes:
    if vtype == STRING:
        b = v.encode() if isinstance(v, str) else bytes(v)
        return struct.pack("<Q", len(b)) + b
    if vtype == ARRAY:
        etype, items = v
        return struct.pack("<IQ", etype, len(items)) + b"".join(_value(etype, x) for x in items)
    return struct.pack(_SCALAR[vtype], v)


def write_gguf(path, metadata, tensors, alignment: int = 32, version: int = 3,
               offsets=None) -> None:
    """Writes a GGUF file.

    metadata: [(key, value_type, value)]; an ARRAY value is (element_type, items).
    tensors:  [(name, ggml_type, dims, data)], dims in GGUF order (dims[0] =
              row length); data is bytes, or (n_bytes, fn) with fn(f) writing
              exactly n_bytes to the open file (large synthetic models).  Data
              is laid out in order, each tensor on an `alignment` boundary;
              `offsets` replaces the relative offsets written in the table
              (malformed files).
    """
    def size_of(data):
        return data[0] if isinstance(data, tuple) else len(data)

    head = bytearray()
    head += struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(metadata))
    for key, vtype, v in metadata:
        head += _value(STRING, key) + struct.pack("<I", vtype) + _value(vtype, v)
    layout, pos = [], 0  # where each tensor's data goes, relative to the data section
    for _, _, _, data in tensors:
        pos = (pos + alignment - 1) // alignment * alignment
        layout.append(pos)
        pos += size_of(data)
    table = layout if offsets is None else list(offsets)
    for (name, gtype, dims, _), off in zip(tensors, table):
        head += _value(STRING, name) + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", gtype, off)
    head += bytes((-len(head)) % alignment)
    with open(path, "wb") as f:
        f.write(head)
        written = 0
        for (_, _, _, data), off in zip(tensors, layout):
            f.write(bytes(off - written))
            if isinstance(data, tuple):
                start = f.tell()
                data[1](f)
                if f.tell() - start != data[0]:
                    raise ValueError("tensor writer wrote the wrong number of bytes")
            else:
                f.write(data)
            written = off + size_of(data)


class GGUFFile:
    """A parsed GGUF file (nexus_gpu_gguf_open); close() or use as a context manager."""

    def __init__(self, path: str):
        self.L = _native.lib()
        self._h = ctypes.c_void_p()
        _native.check(self.L.nexus_gpu_gguf_open(str(path).encode(), ctypes.byref(self._h)))
        m = _native.GgufModel()
        _native.check(self.L.nexus_gpu_gguf_model(self._h, ctypes.byref(m)))
        self.model = {f: getattr(m, f) for f, _ in m._fields_}
        self.model["architecture"] = m.architecture.decode()
        self.tensors = [self.tensor(i) for i in range(m.tensor_count)]

    def tensor(self, index: int) -> dict:
        t = _native.GgufTensor()
        _native.check(self.L.nexus_gpu_gguf_tensor(self._h, index, ctypes.byref(t)))
        d = {f: getattr(t, f) for f, _ in t._fields_}
        d["name"] = t.name.decode()
        d["dims"] = list(t.dims)[:t.n_dims]
        return d

    def find(self, name: str) -> int:
        idx = ctypes.c_uint64()
        _native.check(self.L.nexus_gpu_gguf_find(self._h, name.encode(), ctypes.byref(idx)))
        return idx.value

    def upload(self, names, device=None, stream=None):
        """Uploads the named tensors into one device image.

        Returns (image, {name: (offset, tensor dict)}): `image` is a torch
        uint8 CUDA tensor that owns the memory; a tensor's device pointer is
        image.data_ptr() + offset."""
        import torch

        idx = [self.find(n) for n in names]
        arr = (ctypes.c_uint64 * max(1, len(idx)))(*idx)
        size = self.L.nexus_gpu_gguf_upload_size(self._h, arr, len(idx))
        image = torch.empty(max(size, 1), dtype=torch.uint8, device=device or "cuda")
        offs = (ctypes.c_uint64 * max(1, len(idx)))()
        st = stream.cuda_stream if stream is not None else torch.cuda.current_stream(image.device).cuda_stream
        _native.check(self.L.nexus_gpu_gguf_upload(self._h, arr, len(idx), image.data_ptr(), image.numel(), offs, st))
        return image, {n: (offs[i], self.tensors[idx[i]]) for i, n in enumerate(names)}

    def close(self) -> None:
        if self._h:
            _native.check(self.L.nexus_gpu_gguf_close(self._h))
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
