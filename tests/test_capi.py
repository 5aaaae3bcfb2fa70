"""The C ABI library: it loads, exports every declared entry point, and the
ctypes mirror of the parameter struct matches the C layout. No GPU needed
(nothing here launches a kernel)."""

from __future__ import annotations

import ctypes
import os
import re
import shutil
import subprocess

import pytest

from conftest import ROOT
from unblend_b200 import _lib

HEADER = os.path.join(ROOT, "include", "unblend_b200.h")


def _declared() -> list[str]:
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^int\s+(unblend_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from unblend_b200.build import build

        build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_declares_entry_points():
    names = _declared()
    assert "unblend_conv2d_f32" in names and "unblend_stft_cac" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert set(_lib.exported_symbols()) <= set(_declared())


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
@pytest.mark.parametrize("ctype,cname", [(_lib.ConvParams, "UnblendConvParams"),
                                         (_lib.AttnParams, "UnblendAttnParams"),
                                         (_lib.GemmGroup, "UnblendGemmGroup"),
                                         (_lib.GemmParams, "UnblendGemmParams")])
def test_param_struct_layout_matches_c(tmp_path, ctype, cname):
    fields = [f for f, _ in ctype._fields_]
    src = tmp_path / "layout.c"
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof({cname}, {f}));' for f in fields)
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "unblend_b200.h"\n'
        f'int main(void) {{\n  printf("size %zu\\n", sizeof({cname}));\n{body}\n  return 0;\n}}\n'
    )
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                        check=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(ctype)
    for f in fields:
        assert int(out[f]) == getattr(ctype, f).offset, f


def test_error_codes_raise():
    with pytest.raises(RuntimeError, match="invalid arguments"):
        _lib.check("unblend_x", _lib.ERR_INVALID)
    with pytest.raises(RuntimeError, match="CUDA out of memory"):
        _lib.check("unblend_x", 2)


def test_noalloc_capacity_matches_header():
    text = open(HEADER).read()
    m = re.search(r"^#define\s+UNBLEND_NOALLOC_MAX_BATCH\s+(\d+)", text, flags=re.M)
    assert m and int(m.group(1)) == _lib.NOALLOC_MAX_BATCH
