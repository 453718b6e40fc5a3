"""The ctypes mirror of the C ABI (``nanovllm_dots_b200/_lib.py``) against the
headers themselves: a small C program, compiled here with the system C
compiler against ``include/*.h``, prints ``sizeof`` of every struct and
``offsetof`` of every field the ctypes structure declares; both must equal
what ctypes computes.  A field added, reordered or retyped on one side only
fails here, on the CPU, before any GPU call could read a shifted pointer."""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess

import pytest

from nanovllm_dots_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
HEADERS = ("dfm.h", "dpe.h", "dllm.h", "dvoc.h")
STRUCTS = ("DfmConfig", "DfmWeights", "DfmBatch", "DpeConfig", "DpeWeights", "DpeBatch",
           "DllmConfig", "DllmWeights", "DllmStep", "DvocConfig", "DvocWeights", "DvocBatch")


def _probe_source() -> str:
    lines = ["#include <stddef.h>", "#include <stdio.h>"]
    lines += [f'#include "{h}"' for h in HEADERS]
    lines.append("int main(void) {")
    for name in STRUCTS:
        lines.append(f'  printf("{name} sizeof %zu\\n", sizeof({name}));')
        for field, _ in getattr(_lib, name)._fields_:
            lines.append(f'  printf("{name} {field} %zu\\n", offsetof({name}, {field}));')
    lines += ["  return 0;", "}"]
    return "\n".join(lines) + "\n"


@pytest.fixture(scope="module")
def c_layout(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    d = tmp_path_factory.mktemp("abi")
    src, exe = d / "probe.c", d / "probe"
    src.write_text(_probe_source())
    subprocess.run([cc, "-std=c11", "-Wall", "-Werror", "-I", INCLUDE, str(src), "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    layout = {}
    for line in out.splitlines():
        struct, key, value = line.split()
        layout[(struct, key)] = int(value)
    return layout


@pytest.mark.parametrize("name", STRUCTS)
def test_ctypes_struct_matches_header(c_layout, name):
    cls = getattr(_lib, name)
    assert ctypes.sizeof(cls) == c_layout[(name, "sizeof")], f"{name}: size"
    for field, _ in cls._fields_:
        assert getattr(cls, field).offset == c_layout[(name, field)], f"{name}.{field}: offset"


def test_headers_declare_no_field_the_mirror_lacks(c_layout):
    """Every struct's last ctypes field ends where the C struct ends (up to
    tail padding), so the header holds no trailing field ctypes omits."""
    for name in STRUCTS:
        cls = getattr(_lib, name)
        field, ftype = cls._fields_[-1]
        end = getattr(cls, field).offset + ctypes.sizeof(ftype)
        align = max(ctypes.alignment(t) for _, t in cls._fields_)
        assert c_layout[(name, "sizeof")] == (end + align - 1) // align * align, name


def test_integration_guide_names_only_exported_functions():
    """The C bindings INTEGRATION.md shows a maintainer call only functions
    the library exports."""
    import re
    with open(os.path.join(ROOT, "INTEGRATION.md")) as f:
        text = f.read()
    names = set(re.findall(r"\b((?:dfm|dpe|dllm|dvoc)_[a-z_0-9]+)", text))
    assert names, "no C function named"
    assert sorted(n for n in names if n not in _lib.EXPORTS) == []
