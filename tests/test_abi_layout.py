"""The ctypes mirrors of the C ABI's structs have the C layout (no GPU): a small C program compiled against
include/gravity_b200.h prints every field offset and the struct sizes, and the ctypes structures must agree."""
import ctypes
import os
import shutil
import subprocess

import pytest

from gravityocr_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _c_layout(struct: str, fields, tmp_path):
    src = tmp_path / "layout.c"
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "gravity_b200.h"', "int main(void) {",
             f'  printf("size %zu\\n", sizeof({struct}));']
    lines += [f'  printf("{f} %zu\\n", offsetof({struct}, {f}));' for f in fields]
    lines += ["  return 0;", "}"]
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return {k: int(v) for k, v in (line.split() for line in out.splitlines())}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
@pytest.mark.parametrize("struct,cls", [("gr_epilogue", L.Epilogue), ("gr_sampling", L.Sampling)])
def test_ctypes_struct_matches_c_layout(struct, cls, tmp_path):
    names = [f[0] for f in cls._fields_]
    c = _c_layout(struct, names, tmp_path)
    assert c["size"] == ctypes.sizeof(cls)
    for n in names:
        assert c[n] == getattr(cls, n).offset, n
