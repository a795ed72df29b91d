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


def test_mqa_params_layout_matches_c_header():
    from deepseek_v4_kernel import indexer
    import ctypes
    fields = "".join(f"F(dsv4b_mqa_logits_params, {n})" for n, _ in indexer.MqaLogitsParams._fields_)
    probe = PROBE.replace('printf("sizeof_params %zu\\nsizeof_meta %zu\\n", sizeof(dsv4b_decode_params), '
                          'sizeof(dsv4b_sched_meta));',
                          'printf("sizeof_params %zu\\n", sizeof(dsv4b_mqa_logits_params));')
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(src, "w").write(probe.replace("%FIELDS%", fields))
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), src, "-o", exe], check=True)
        lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.split() for l in lines if l.strip())
    assert int(got["sizeof_params"]) == ctypes.sizeof(indexer.MqaLogitsParams)
    for n, _ in indexer.MqaLogitsParams._fields_:
        assert int(got[n]) == getattr(indexer.MqaLogitsParams, n).offset, n


def test_writer_and_indexer_reject_bad_arguments_without_a_gpu():
    """Argument checks run before any CUDA call: these return
    DSV4B_ERR_INVALID_ARGUMENT (-1) / DSV4B_ERR_UNSUPPORTED (-2) here."""
    import ctypes
    from deepseek_v4_kernel import _lib, indexer
    lib = _lib.lib
    buf = ctypes.create_string_buffer(1 << 16)
    a = (ctypes.addressof(buf) + 15) & ~15          # a 16-byte aligned host address (never dereferenced)
    # writer: bad layout, null cache, misaligned stride, bad slot width, negative n
    assert lib.dsv4b_kv_cache_write(5, a, 512, a, 64, a, 8, 1, a, 1, 64, 64 * 656, 656, None) == -1
    assert lib.dsv4b_kv_cache_write(0, a, 512, a, 64, a, 8, 1, None, 1, 64, 64 * 656, 656, None) == -1
    assert lib.dsv4b_kv_cache_write(0, a, 512, a, 64, a, 8, 1, a, 1, 64, 64 * 656 + 8, 656, None) == -1
    assert lib.dsv4b_kv_cache_write(0, a, 512, a, 64, a, 2, 1, a, 1, 64, 64 * 656, 656, None) == -1
    assert lib.dsv4b_kv_cache_write(0, a, 512, a, 64, a, 8, -1, a, 1, 64, 64 * 656, 656, None) == -1
    assert lib.dsv4b_kv_cache_write(1, a, 512, a + 2, 512, a, 8, 4, a, 1, 64, 64 * 584, 0, None) == -1  # rope misaligned
    assert lib.dsv4b_kv_cache_write(0, a, 500, a, 64, a, 8, 4, a, 1, 64, 64 * 656, 656, None) == -1    # stride % 8
    assert lib.dsv4b_kv_cache_write(0, a, 512, a, 64, a, 8, 0, a, 1, 64, 64 * 656, 656, None) == 0     # n = 0: nothing to do
    flags = ctypes.c_int()
    assert lib.dsv4b_kv_cache_write_status(None, None) == -1
    assert lib.dsv4b_kv_write_selftest(None, 1, a, None) == -1
    # indexer
    assert lib.dsv4b_mqa_logits_metadata(None, 4, 148, a, None) == -1
    assert lib.dsv4b_mqa_logits_metadata(a, 0, 148, a, None) == -1
    assert lib.dsv4b_mqa_logits_metadata(a, 4, 0, a, None) == -1
    assert lib.dsv4b_mqa_logits_metadata(a, 20000, 148, a, None) == -1

    def params(**kw):
        p = indexer.MqaLogitsParams(4, 1, 64, 128, a, a, 8, 64, 64 * 132, a, a, a, 4, a, 1024, 1024, 1)
        for k, v in kw.items():
            setattr(p, k, v)
        return p

    ok = params()
    for bad, rc in ((params(d=64), -1), (params(h=48), -2), (params(next_n=8), -2), (params(page_block_size=48), -2),
                    (params(stride_kv_block=64 * 132 + 8), -1), (params(stride_kv_block=64 * 100), -1),
                    (params(q=a + 4), -1), (params(logits=None), -1), (params(stride_logits=100), -1),
                    (params(b=0), -1)):
        assert lib.dsv4b_fp8_paged_mqa_logits(ctypes.byref(bad), a, 148, None) == rc
    assert lib.dsv4b_fp8_paged_mqa_logits(ctypes.byref(ok), None, 148, None) == -1
    assert lib.dsv4b_fp8_paged_mqa_logits(ctypes.byref(ok), a, 0, None) == -1
    assert lib.dsv4b_mqa_logits_status(None, None) == -1
