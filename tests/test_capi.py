"""The C-ABI library loads and exports every entry point include/*.h declares (no GPU needed)."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "train-model-template_b200", "libmxmlp.so")


def declared():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(mxm_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared()
    for n in ("mxm_version", "mxm_quant_rows", "mxm_quant_cols", "mxm_gemm"):
        assert n in names


def test_library_exports_all_declared_symbols():
    assert os.path.exists(LIB), "build the library first (train-model-template_b200/build.py)"
    lib = ctypes.CDLL(LIB)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_version_and_errors_without_gpu():
    import _mxlib
    assert _mxlib.version() == 1
    # argument checks run before any CUDA call: a bad shape is rejected with a message
    with pytest.raises(_mxlib.MXError) as ei:
        _mxlib.call("mxm_quant_rows", ctypes.c_void_p(16), 4, 100, 100, ctypes.c_void_p(16), 100,
                    ctypes.c_void_p(16), None)
    assert "K % 128" in str(ei.value)
    with pytest.raises(_mxlib.MXError):
        _mxlib.call("mxm_gemm", None, 128, None, None, 128, None, 128, 256, 128, None, 256, None)
