"""The ctypes mirrors of the header's structs have the C compiler's layout
(size and every field offset), so Python callers pass the same bytes a C
caller would."""
import ctypes
import os
import shutil
import subprocess

import pytest

from nexusllm_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
@pytest.mark.parametrize("cname,py", [("NexusGpuStackTask", _native.StackTask),
                                      ("NexusGpuStackTaskEx", _native.StackTaskEx)])
def test_struct_layout_matches_the_header(tmp_path, cname, py):
    fields = [f for f, _ in py._fields_]
    body = "".join(f'    printf("%zu ", offsetof({cname}, {f}));\n' for f in fields)
    src = tmp_path / "layout.c"
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "nexus_gpu.h"\nint main(void) {\n'
                   f'    printf("%zu ", sizeof({cname}));\n{body}    return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    want = [ctypes.sizeof(py)] + [getattr(py, f).offset for f in fields]
    assert got == want
