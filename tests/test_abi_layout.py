"""The ctypes mirrors of the C ABI's structs have the C compiler's layout.

A small C program including include/vorotracing_b200.h prints sizeof and
offsetof of every struct field; the ctypes Structure classes the Python layer
passes by pointer must agree field by field (a mismatch would hand the
kernels shifted pointers).  Runs on CPU with gcc.
"""
import ctypes as C
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

STRUCTS = {
    "vt_scene": ("vorotracing_b200._lib", "VtScene"),
    "vt_debug": ("vorotracing_b200._lib", "VtDebug"),
    "vt_path": ("vorotracing_b200._lib", "VtPath"),
    "vt_camera": ("vorotracing_b200.cameras", "VtCamera"),
    "vt_peer_grads": ("vorotracing_b200._lib", "VtPeerGrads"),
}


def _c_layout(tmp_path):
    import importlib

    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "vorotracing_b200.h"',
             "int main(void) {"]
    for cname, (mod, cls) in STRUCTS.items():
        py = getattr(importlib.import_module(mod), cls)
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)])
    out = subprocess.check_output([str(exe)], text=True).split("\n")
    got = {}
    for line in out:
        if line.strip():
            *key, val = line.split()
            got[tuple(key)] = int(val)
    return got


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_ctypes_structs_match_the_header(tmp_path):
    import importlib

    layout = _c_layout(tmp_path)
    for cname, (mod, cls) in STRUCTS.items():
        py = getattr(importlib.import_module(mod), cls)
        assert C.sizeof(py) == layout[(cname, "size")], cname
        for fname, _ in py._fields_:
            assert getattr(py, fname).offset == layout[(cname, fname)], (cname, fname)
