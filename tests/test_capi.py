"""CPU: the C-ABI library loads and exports every entry point the header declares."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    hdr = open(os.path.join(ROOT, "include", "qvggt_b200.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(qvggt_\w+)\s*\(", hdr)))


def test_header_declares_entry_points():
    names = _declared()
    assert "qvggt_w4a16_gemm" in names and "qvggt_attention" in names
    assert len(names) >= 18


def test_library_exports_every_declared_symbol():
    from qvggt_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built")
    import ctypes
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing
    # the ctypes signature table covers the header exactly
    assert sorted(_lib.SIGNATURES) == _declared()


def test_library_reports_errors_without_gpu():
    """Calls that fail argument checks return an error code and a message
    without touching a device."""
    from qvggt_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built")
    lib = _lib.load()
    assert lib.qvggt_version() >= 100
    rc = lib.qvggt_w4a16_gemv(None, None, None, None, None, None, 17, 128, 128, 8, 128, None)
    assert rc == 2
    assert b"m=17" in lib.qvggt_last_error()
    rc = lib.qvggt_set_wait_timeout_ns(0)
    assert rc == 1
