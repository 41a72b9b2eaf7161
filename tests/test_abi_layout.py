"""The ctypes mirrors of the C ABI's structs have the header's layout: a C
program compiled against include/kvr_b200.h prints every struct's size and
field offsets, and the ctypes classes must agree field by field (a field added
on one side only would shift every field after it)."""

import os
import shutil
import subprocess

import pytest

from budgeted_kv_cache_repair_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STRUCTS = {"kvr_layer_weights": _lib.LayerWeights, "kvr_model": _lib.Model,
           "kvr_refresh_request": _lib.RefreshRequest, "kvr_linear_segment": _lib.LinearSegment}


def test_ctypes_structs_match_the_header(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    body = []
    for cname, mirror in STRUCTS.items():
        body.append(f'printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for field, _ in mirror._fields_:
            body.append(f'printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    src = tmp_path / "layout.c"
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "kvr_b200.h"\nint main(void) {\n'
                   + "\n".join(body) + "\nreturn 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    printed = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        cname, field, value = line.split()
        printed[(cname, field)] = int(value)
    import ctypes

    for cname, mirror in STRUCTS.items():
        assert printed[(cname, "sizeof")] == ctypes.sizeof(mirror), cname
        for field, _ in mirror._fields_:
            assert printed[(cname, field)] == getattr(mirror, field).offset, (cname, field)
