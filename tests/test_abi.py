"""CPU: the C-ABI library loads, exports every symbol include/dsv4b.h
declares, and the ctypes structures match the C layout (checked against a
gcc-compiled probe of the header).  No compute calls (no GPU here)."""
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dsv4b.h")


def _declared():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"DSV4B_API\s+[\w\s\*]+?\b(dsv4b_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    from deepseek_v4_kernel import _lib
    names = _declared()
    assert len(names) >= 10
    assert sorted(_lib.EXPORTED) == names
    for n in names:
        assert hasattr(_lib.lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (dsv4b_\w+)", out))
    assert set(names) <= exported


def test_status_strings_and_version():
    from deepseek_v4_kernel import _lib
    assert _lib.lib.dsv4b_version() >= 100
    for code in _lib.STATUS:
        assert _lib.lib.dsv4b_status_string(code)
    assert _lib.lib.dsv4b_workspace_bytes(32, 1, 64, 148) > 0
    assert _lib.lib.dsv4b_workspace_bytes(0, 1, 64, 148) == 0


def test_invalid_arguments_fail_before_touching_a_gpu():
    import ctypes
    from deepseek_v4_kernel import _lib
    p = _lib.DecodeParams()          # all zero: b = 0
    assert _lib.lib.dsv4b_sparse_decode(ctypes.byref(p), None, None, 1, None, 0, None) == -1
    assert _lib.lib.dsv4b_sparse_decode(None, None, None, 1, None, 0, None) == -1
    assert _lib.lib.dsv4b_gather_dequant(7, None, 1, 1, 0, 0, None, 0, None, None) == -1


PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "dsv4b.h"
#define F(s, f) printf(#f " %zu\n", offsetof(s, f));
int main(void) {
  printf("sizeof_params %zu\nsizeof_meta %zu\n", sizeof(dsv4b_decode_params), sizeof(dsv4b_sched_meta));
  %FIELDS%
  return 0;
}
"""


def test_ctypes_layout_matches_c_header():
    from deepseek_v4_kernel import _lib
    fields = "".join(f"F(dsv4b_decode_params, {n})" for n, _ in _lib.DecodeParams._fields_)
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(src, "w").write(PROBE.replace("%FIELDS%", fields))
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), src, "-o", exe], check=True)
        lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.split() for l in lines if l.strip())
    import ctypes
    assert int(got["sizeof_params"]) == ctypes.sizeof(_lib.DecodeParams)
    assert int(got["sizeof_meta"]) == ctypes.sizeof(_lib.SchedMeta) == 32
    for n, _ in _lib.DecodeParams._fields_:
        assert int(got[n]) == getattr(_lib.DecodeParams, n).offset, n
