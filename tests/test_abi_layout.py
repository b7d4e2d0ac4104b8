"""The ctypes mirrors of the C-ABI structs have the header's layout.

A small C program compiled with gcc against include/int8_linear_b200.h prints the size
and every field offset of struct i8l_tile and struct i8l_peer_comm; the ctypes
structures in int8_linear/_native.py must agree field by field (and so must any
binding written from the header, e.g. a cgo or JNI stub).  CPU only.
"""

from __future__ import annotations

import ctypes
import shutil
import subprocess
from pathlib import Path

import pytest

from int8_linear import _native

ROOT = Path(__file__).resolve().parent.parent
STRUCTS = {
    "i8l_tile": (_native.I8LTile, [f for f, _ in _native.I8LTile._fields_]),
    "i8l_peer_comm": (_native.I8LPeerComm, [f for f, _ in _native.I8LPeerComm._fields_]),
}


def _c_layout(tmp_path: Path) -> dict[str, dict[str, int]]:
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "int8_linear_b200.h"', "int main(void) {"]
    for name, (_, fields) in STRUCTS.items():
        lines.append(f'  printf("{name} sizeof %zu\\n", sizeof(struct {name}));')
        for f in fields:
            lines.append(f'  printf("{name} {f} %zu\\n", offsetof(struct {name}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    layout: dict[str, dict[str, int]] = {}
    for line in out.splitlines():
        struct, field, value = line.split()
        layout.setdefault(struct, {})[field] = int(value)
    return layout


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_ctypes_structs_match_the_header(tmp_path):
    layout = _c_layout(tmp_path)
    for name, (cls, fields) in STRUCTS.items():
        assert layout[name]["sizeof"] == ctypes.sizeof(cls), name
        for f in fields:
            assert layout[name][f] == getattr(cls, f).offset, (name, f)
