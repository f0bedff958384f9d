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


def test_noalloc_chunking_fits_the_fixed_scratch():
    """mxm_coldot_noalloc's row chunking (host arithmetic, no GPU): mxm_coldot's chunking on a B200-sized
    device, fewer and taller chunks where the partials would not fit the 16 MiB scratch."""
    import _mxlib
    def chunks(T, K, n, sms):
        rpc, nch = ctypes.c_int(0), ctypes.c_int(0)
        _mxlib.call("mxm_coldot_noalloc_chunks", T, K, n, sms, ctypes.byref(rpc), ctypes.byref(nch))
        return rpc.value, nch.value
    for T, K, n in ((16384, 2048, 16), (142336, 6144, 64), (77, 64, 16), (20000, 2048, 64)):
        for sms in (148, 1024, 4096):
            rpc, nch = chunks(T, K, n, sms)
            assert rpc % 64 == 0 and rpc * nch >= T and (nch - 1) * rpc < T
            assert nch * K * n * 4 <= 16 << 20
        a, b = ctypes.c_int(0), ctypes.c_int(0)
        _mxlib.call("mxm_coldot_chunks", T, K, ctypes.byref(a), ctypes.byref(b))
        assert chunks(T, K, n, 148) == (a.value, b.value)   # below the cap: the regular chunking
    assert chunks(20000, 2048, 64, 1024)[1] == 32             # the cap: 16 MiB / (2048 * 64 * 4 B)
    with pytest.raises(_mxlib.MXError):
        chunks(128, 131072, 64, 148)


def _bwd_plan(T, N, r, sms=148):
    """The backward epilogue's partition restated (host arithmetic): row blocks of 256 rows (rank 16) or
    176 (rank 32), 32-column tiles column-fastest, contiguous runs of ceil(items / SMs) per CTA."""
    sb = 256 if r == 16 else 176
    nsb = -(-(-(-T // 128) * 128) // sb)
    nt = N // 32
    items = nsb * nt
    per = -(-items // sms)
    slots = max(((b + 1) * nt - 1) // per - (b * nt) // per + 1 for b in range(nsb))
    return sb, max(slots, 1)


def test_bwd_partition_and_argument_checks_without_gpu():
    """mxm_mlp_bwd_partitions agrees with the restated plan, and mxm_mlp_bwd_epilogue rejects a gu_lora
    flag it cannot honour before touching the device."""
    import _mxlib
    for T, N, r in ((1, 128, 16), (300, 6144, 16), (16384, 6144, 16), (142336, 6144, 16), (10752, 3584, 16),
                    (2049, 3584, 32), (16384, 6144, 32)):
        assert _mxlib.mlp_bwd_partitions(T, N, r) == _bwd_plan(T, N, r), (T, N, r)
    p = ctypes.c_void_p(256)
    for r, gu_lora in ((32, 1), (16, 2)):
        sb, ncg = _bwd_plan(300, 6144, r)
        with pytest.raises(_mxlib.MXError) as ei:
            _mxlib.call("mxm_mlp_bwd_epilogue", p, p, p, p, p, p, p, 300, 6144, r, 2.0, 2.0, gu_lora, None, None, p, p,
                        p, p, sb, ncg, None)
        assert "gu_lora" in str(ei.value) or "rank-16" in str(ei.value)
