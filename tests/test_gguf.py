"""The GGUF parser (nexus_gpu_gguf_open / _model / _tensor / _find) against
NexusLLM's own loader (UniversalModelLoader::load_gguf, src/model_loader.cpp:
416-836), recorded in tests/golden/gguf_ref.json from the synthetic files of
tests/gguf_cases.py (and re-run live when oracle/_ref/libnexus_ref_gguf.so is
built).  Parsing is host-only, so all of this runs without a GPU.

Same as the reference: metadata (keys, defaults, inferred dimensions), which
names resolve (aliases, tied LM head), dims and the data each tensor points
at.  Different on purpose (include/nexus_gpu.h): one-to-one ggml type mapping,
true byte sizes, tensors running past the end of the file skipped, nested
metadata arrays parsed."""
import ctypes
import json
import os
import struct

import numpy as np
import pytest

import gguf_cases
import oracle
from nexusllm_b200 import _native, gguf

HERE = os.path.dirname(os.path.abspath(__file__))
FIELDS = ["architecture", "vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
          "num_attention_heads", "num_key_value_heads", "max_position_embeddings", "rms_norm_eps", "rope_theta",
          "is_moe", "num_experts", "num_experts_per_tok"]
# tensors that start inside the file and run past its end (names that resolve
# to them, and their count): the reference registers them, this parser skips them
RUNS_PAST_END = {"fallbacks": {"model.layers.2.self_attn.v_proj.weight", "layers.2.wv"}}
RUNS_PAST_END_COUNT = {"fallbacks": 1}


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(HERE, "golden", "gguf_ref.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    return gguf_cases.build(str(tmp_path_factory.mktemp("gguf")))


def _f32(v):
    return struct.unpack("<I", struct.pack("<f", v))[0]


def _ours(path, names):
    with gguf.GGUFFile(path) as f:
        out = []
        for n in names:
            try:
                out.append(f.tensors[f.find(n)])
            except _native.NexusGpuError:
                out.append(None)
        return f.model, f.tensors, out


def test_fixture_covers_every_case(golden):
    assert set(golden) == set(gguf_cases.CASES)
    assert golden["nested_array"]["status"] == -3          # the reference cannot parse it
    assert all(golden[c]["status"] == 0 for c in ("reference_fixture", "mixed_types", "fallbacks"))


@pytest.mark.parametrize("case", ["reference_fixture", "mixed_types", "fallbacks"])
def test_metadata_matches_reference(golden, files, case):
    model, _, _ = _ours(files[case][0], [])
    ref = golden[case]["model"]
    for k in FIELDS:
        if k == "rms_norm_eps":
            assert _f32(model[k]) == _f32(ref[k]), k
        else:
            assert model[k] == ref[k], (k, model[k], ref[k])
    assert model["tensor_count"] + RUNS_PAST_END_COUNT.get(case, 0) == ref["loaded_tensor_count"]


def test_nested_arrays_parse(golden, files):
    """The reference fails on an array of arrays; this parser skips it and reads
    the same metadata as from the file without it."""
    model, _, _ = _ours(files["nested_array"][0], [])
    ref = golden["mixed_types"]["model"]
    for k in FIELDS:
        assert (_f32(model[k]) == _f32(ref[k])) if k == "rms_norm_eps" else (model[k] == ref[k]), k


@pytest.mark.parametrize("case", ["reference_fixture", "mixed_types", "fallbacks"])
def test_tensors_match_reference(golden, files, case):
    path, written = files[case]
    g = golden[case]
    _, _, ours = _ours(path, g["names"])
    raw = open(path, "rb").read()
    types = {t[0]: t[1] for t in written}
    sizes = {t[0]: len(t[3]) for t in written}
    for name, ref, mine, hb in zip(g["names"], g["tensors"], ours, g["hash_bytes"]):
        if name in RUNS_PAST_END.get(case, ()):
            assert ref["found"] and mine is None, name
            continue
        assert bool(ref["found"]) == (mine is not None), name
        if mine is None:
            continue
        assert mine["dims"] == ref["dims"], name
        assert mine["cols"] == mine["dims"][0] and mine["rows"] == int(np.prod(mine["dims"][1:])), name
        gt = types[mine["name"]]
        if gt in gguf_cases.REFERENCE_REMAPS:  # the reference re-labels this type; we do not
            assert ref["dtype"] == gguf_cases.REFERENCE_REMAPS[gt] and mine["dtype"] == -1, name
        else:
            assert mine["dtype"] == ref["dtype"], name
        assert mine["bytes"] == sizes[mine["name"]] == hb, name        # true block sizes
        data = raw[mine["file_offset"]:mine["file_offset"] + mine["bytes"]]
        assert oracle.fnv1a(data) == ref["fnv"], name                 # the same data the reference maps


def test_reference_over_counts_quantized_sizes(golden):
    """TensorShape::total_bytes (include/nexus_common.hpp:262-281) counts Q4_0
    at 5 bits and Q8_0 at 9 bits per weight; the block sizes are 4.5 and 8.5."""
    g = golden["reference_fixture"]
    by = dict(zip(g["names"], g["tensors"]))
    assert by["blk.0.ffn_gate.weight"]["byte_size"] == 64 * 128 * 5 // 8      # file holds 64*128/32*18
    assert by["blk.0.attn_q.weight"]["byte_size"] == 64 * 64 * 9 // 8
    assert 64 * 128 // 32 * 18 != 64 * 128 * 5 // 8


def test_lm_head_rows_are_the_vocabulary(files):
    """forward_pass.cpp:581 takes dims[0] of the LM head as the vocabulary
    size; it is the row length.  rows = dims[1]."""
    with gguf.GGUFFile(files["mixed_types"][0]) as f:
        t = f.tensors[f.find("lm_head")]
        assert t["name"] == "output.weight" and t["rows"] == 1000 and t["cols"] == 512 and t["served"] == 1


def test_tied_lm_head_and_aliases(files):
    with gguf.GGUFFile(files["fallbacks"][0]) as f:
        assert f.tensors[f.find("lm_head")]["name"] == "model.embed_tokens.weight"
        assert f.tensors[f.find("output.weight")]["name"] == "model.embed_tokens.weight"
        assert f.tensors[f.find("layers.0.wq")]["name"] == "model.layers.0.self_attn.q_proj.weight"
        assert f.tensors[f.find("blk.0.attn_q.weight")]["name"] == "model.layers.0.self_attn.q_proj.weight"
        assert f.model["skipped"] == 2
        with pytest.raises(_native.NexusGpuError):
            f.find("layers.1.wk")                                    # starts past the end of the file


@pytest.mark.skipif(not oracle.reference_gguf_available(), reason="reference loader not built")
def test_live_reference_agrees_with_the_fixture(golden, files):
    for case, (path, _) in files.items():
        g = golden[case]
        st, model, res = oracle.reference_gguf_load(path, g["names"], g["hash_bytes"])
        assert st == g["status"] and model == g["model"] and res == g["tensors"], case


def test_open_rejects_malformed_files(tmp_path):
    L = _native.lib()
    h = ctypes.c_void_p()
    bad = -3  # NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED
    assert L.nexus_gpu_gguf_open(str(tmp_path / "missing.gguf").encode(), ctypes.byref(h)) == bad
    p = tmp_path / "t.gguf"
    gguf_cases.reference_fixture(str(p))
    good = p.read_bytes()
    for name, data in [("magic", b"GGUX" + good[4:]), ("v1", good[:4] + struct.pack("<I", 1) + good[8:]),
                       ("truncated", good[:200]), ("empty", b""),
                       ("kv_type", good[:52] + struct.pack("<I", 77) + good[56:])]:  # first key's value type
        q = tmp_path / f"{name}.gguf"
        q.write_bytes(data)
        assert L.nexus_gpu_gguf_open(str(q).encode(), ctypes.byref(h)) == bad, name
        assert h.value is None
    assert L.nexus_gpu_gguf_open(None, ctypes.byref(h)) == -9


@pytest.mark.parametrize("vtype,value,ok", [
    (gguf.U32, 0, True),             # 0 means the default, 32 (model_loader.cpp:640)
    (gguf.U32, 64, True),
    (gguf.U64, 1 << 31, True),
    (gguf.U64, 1 << 32, False),      # the reference's 32-bit cast would make this 0
    (gguf.U64, 1 << 40, False),
    (gguf.U32, 48, False),           # not a power of two: the reference's mask rounding differs
    (gguf.U32, 3, False),
])
def test_open_checks_the_alignment(tmp_path, vtype, value, ok):
    """general.alignment must be a power of two up to 2^31; anything else is
    refused with a message instead of a division by zero or a wrong offset."""
    L = _native.lib()
    p = tmp_path / "a.gguf"
    norm = struct.pack("<4f", 1.0, 1.0, 1.0, 1.0)
    gguf.write_gguf(str(p), [("general.architecture", gguf.STRING, "llama"), ("general.alignment", vtype, value)],
                    [("blk.0.attn_norm.weight", gguf.GGML_F32, [4], norm)], alignment=32)
    h = ctypes.c_void_p()
    rc = L.nexus_gpu_gguf_open(str(p).encode(), ctypes.byref(h))
    if ok:
        assert rc == 0, L.nexus_gpu_last_error()
        assert L.nexus_gpu_gguf_close(h) == 0
    else:
        assert rc == -3 and h.value is None
        assert b"general.alignment" in L.nexus_gpu_last_error()


def test_upload_checks_before_touching_a_device(files):
    """Refusals that need no device: an unmapped type, a small buffer."""
    with gguf.GGUFFile(files["mixed_types"][0]) as f:
        L = f.L
        q41 = f.find("blk.0.attn_k.weight")                        # Q4_1: no NexusLLM DataType
        q40 = f.find("blk.0.attn_q.weight")
        arr = (ctypes.c_uint64 * 2)(q40, q41)
        offs = (ctypes.c_uint64 * 2)()
        assert L.nexus_gpu_gguf_upload(f._h, arr, 2, None, 0, offs, None) == -3
        one = (ctypes.c_uint64 * 1)(q40)
        need = L.nexus_gpu_gguf_upload_size(f._h, one, 1)
        assert need == f.tensors[q40]["bytes"]
        assert L.nexus_gpu_gguf_upload(f._h, one, 1, 16, need - 1, offs, None) == -102
        two = (ctypes.c_uint64 * 2)(q40, f.find("blk.0.ffn_gate.weight"))
        size = L.nexus_gpu_gguf_upload_size(f._h, two, 2)
        assert size == (f.tensors[q40]["bytes"] + 255) // 256 * 256 + f.tensors[two[1]]["bytes"]
        assert L.nexus_gpu_gguf_upload_size(f._h, (ctypes.c_uint64 * 1)(10 ** 6), 1) == 0
