"""The ctypes mirrors of the C-ABI parameter structs match include/dsa_b200.h (CPU).

A C program compiled with the system compiler from the header prints the size of every
parameter struct and the offset of each field the Python binding declares; a field added to
one side only, or in a different order, shows up here instead of as a wrong pointer on the
GPU.
"""
import ctypes
import os
import shutil
import subprocess

import pytest

from dsa_triton_ascend_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STRUCTS = {
    "DsaSfaFwdParams": _lib.SfaFwdParams,
    "DsaSfaBwdParams": _lib.SfaBwdParams,
    "DsaLiParams": _lib.LiParams,
    "DsaSliParams": _lib.SliParams,
    "DsaDenseIndexerParams": _lib.DenseIndexerParams,
}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_ctypes_structs_match_the_header(tmp_path):
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "dsa_b200.h"', 'int main(void) {']
    for cname, py in STRUCTS.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ['  return 0;', '}']
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l.strip()}
    for cname, py in STRUCTS.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for field, _ in py._fields_:
            assert got[(cname, field)] == getattr(py, field).offset, (cname, field)
