"""The C-ABI library loads without a GPU and exports every function that
include/*.h declares.  No compute calls (CPU only)."""
import ctypes
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(mb_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("mb_quantize", "mb_quantize_extract_outliers", "mb_dequantize", "mb_pack_2bit",
              "mb_unpack_2bit", "mb_pack_4bit", "mb_unpack_4bit", "mb_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from memboost_b200 import _C
    lib = ctypes.CDLL(_C.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_library_is_sm100a_only_build():
    from memboost_b200 import _C
    assert "sm_100a" in _C.version()


def test_workspace_size_query_needs_no_gpu():
    from memboost_b200 import _C
    n1 = _C._lib.mb_quantize_workspace_size(4096, 4096)
    n2 = _C._lib.mb_quantize_workspace_size(4096, 11008)
    assert 0 < n1 < n2
    assert _C._lib.mb_quantize_workspace_size(0, 16) == 0


def test_argument_errors_without_gpu():
    # invalid sizes are rejected before any CUDA call
    from memboost_b200 import _C
    st = _C._lib.mb_pack_2bit(None, 15, None, None)
    assert st == 1 and b"multiple of 16" in _C._lib.mb_last_error()
    st = _C._lib.mb_unpack_4bit(None, 1, 9, None, None)
    assert st == 1 and b"too large" in _C._lib.mb_last_error()
    st = _C._lib.mb_quantize(None, 4, 4, 0.1, None, 0, *([None] * 10), None, 0, None)
    assert st == 1
