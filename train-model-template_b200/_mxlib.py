"""ctypes binding of the native library libmxmlp.so (C ABI in include/mxmlp.h).

The library is required: importing this module raises ImportError when it is missing or does
not load, and every call checks the returned status and raises RuntimeError with the library's
message.  There is no CPU or Python fallback for any kernel.
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmxmlp.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"MXFP8 native library not built: {LIB_PATH} is missing (run build.py)")
try:
    _lib = ctypes.CDLL(LIB_PATH)
except OSError as e:  # pragma: no cover - depends on the machine
    raise ImportError(f"MXFP8 native library failed to load: {e}") from e

_vp, _i64, _int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int


class GroupBranch(ctypes.Structure):
    """mxm_group_branch (include/mxmlp.h): one branch of a linear group's backward."""
    _fields_ = [("dy", _vp), ("ldy", _i64), ("N", _i64), ("xa", _vp), ("ldxa", _i64), ("Bt", _vp), ("r", _int),
                ("scale", ctypes.c_float), ("dxa_out", _vp), ("ld_dxa", _i64), ("dB_out", _vp)]


# name -> argument types (all return int status unless listed in _RESTYPE)
_SIGS = {
    "mxm_version": [],
    "mxm_last_error": [],
    "mxm_device_error": [ctypes.POINTER(ctypes.c_int), _int],
    "mxm_selftest_wait": [_i64, _vp],
    "mxm_num_sms": [],
    "mxm_launch_count": [],
    "mxm_quant_rows": [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp],
    "mxm_quant_cols": [_vp, _i64, _i64, _i64, _vp, _vp, _vp],
    "mxm_quant_both": [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp],
    "mxm_gemm": [_vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp],
    "mxm_gemm_lora": [_vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _int, _vp, _i64, _vp],
    "mxm_gemm_glu_partition": [_i64, _i64, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                               ctypes.POINTER(ctypes.c_int)],
    "mxm_gemm_glu": [_vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _int, ctypes.c_float,
                     ctypes.c_float, _vp, _vp, _vp, _vp, _vp],
    "mxm_mlp_fwd_partitions": [_i64, _i64, _int, ctypes.POINTER(ctypes.c_int)],
    "mxm_mlp_fwd_epilogue": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, ctypes.c_float, ctypes.c_float, _vp, _vp,
                             _vp, _vp, _int, _vp],
    "mxm_mlp_bwd_partitions": [_i64, _i64, _int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)],
    "mxm_mlp_bwd_epilogue": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, ctypes.c_float, ctypes.c_float,
                             _int, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _vp],
    "mxm_mlp_bwd_reduce": [_vp, _vp, _vp, _vp, _i64, _i64, _int, ctypes.c_float, ctypes.c_float, _int, _int, _vp,
                           _vp, _vp, _vp, _vp, _vp],
    "mxm_rowdot": [_vp, _i64, _vp, _i64, _i64, _int, ctypes.c_float, _vp, _i64, _vp],
    "mxm_rowdot_quant": [_vp, _i64, _vp, _i64, _i64, _int, ctypes.c_float, _vp, _i64, _vp, _i64, _vp, _vp],
    "mxm_coldot_chunks": [_i64, _i64, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)],
    "mxm_coldot": [_vp, _i64, _vp, _i64, _i64, _i64, _int, ctypes.c_float, _int, _vp, _int, _int, _vp, _int, _vp],
    "mxm_quant_rows_into": [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _vp],
    "mxm_lora_bwd": [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _int, ctypes.c_float, _vp, _i64, _vp, _i64, _i64, _vp, _i64,
                     _vp, _vp, _int, _int, _vp],
    "mxm_res_lora": [_vp, _vp, _vp, _i64, _vp, _i64, _i64, _int, ctypes.c_float, _vp, _vp],
    "mxm_lora_prep": [_vp, _vp, _vp, _vp, _vp, _vp, _int, _i64, _i64, _int, ctypes.c_float, _vp, _vp],
    "mxm_group_lora_bwd": [_i64, _int, ctypes.POINTER(GroupBranch), _vp, _i64, _vp, _i64, _vp, _i64, _vp],
    "mxm_coldot_noalloc": [_vp, _i64, _vp, _i64, _i64, _i64, _int, ctypes.c_float, _int, _vp, _vp],
    "mxm_coldot_noalloc_chunks": [_i64, _i64, _int, _int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)],
}
_RESTYPE = {"mxm_last_error": ctypes.c_char_p, "mxm_launch_count": ctypes.c_ulonglong}

for _name, _args in _SIGS.items():
    _f = getattr(_lib, _name)
    _f.argtypes = _args
    _f.restype = _RESTYPE.get(_name, ctypes.c_int)

EXPORTED = tuple(_SIGS)


class MXError(RuntimeError):
    """A native call returned a non-zero status."""

    def __init__(self, fn, status, msg):
        super().__init__(f"{fn} failed (status {status}): {msg}")
        self.status = status


def last_error():
    m = _lib.mxm_last_error()
    return m.decode() if m else ""


def call(name, *args):
    st = getattr(_lib, name)(*args)
    if st != 0:
        raise MXError(name, st, last_error())
    return st


def version():
    return _lib.mxm_version()


MXM_ERR_DEVICE = -4


def device_error(clear=True):
    """The device-side error code of the current device (0 = none; a kernel gave up a bounded wait
    otherwise), cleared when `clear`.  Synchronizes the device."""
    c = ctypes.c_int(0)
    st = _lib.mxm_device_error(ctypes.byref(c), 1 if clear else 0)
    if st not in (0, MXM_ERR_DEVICE):
        raise MXError("mxm_device_error", st, last_error())
    return c.value


def launch_count():
    """Kernels launched by the native library so far in this process."""
    return int(_lib.mxm_launch_count())


def num_sms():
    return _lib.mxm_num_sms()


def ctypes_ref(x):
    """ctypes.byref, for the entry points that return values through int pointers."""
    return ctypes.byref(x)


def ptr(t):
    """Device pointer of a tensor as an integer for a void* argument (None -> NULL)."""
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t=None):
    """The current torch CUDA stream handle of t's device (the current device for None), for a void*."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index if t is not None and t.device.index is not None
                           else torch.cuda.current_device())
    dev = t.device if t is not None else None
    return torch.cuda.current_stream(dev).cuda_stream


# ---- partition queries: pure functions of the shape and the device, asked once per shape
_QUERY = {}


def _query(name, *args, n_out):
    key = (name, torch.cuda.current_device() if torch.cuda.is_available() else -1) + args
    hit = _QUERY.get(key)
    if hit is None:
        outs = [ctypes.c_int(0) for _ in range(n_out)]
        call(name, *args, *[ctypes.byref(o) for o in outs])
        hit = _QUERY[key] = tuple(o.value for o in outs)
    return hit


def coldot_chunks(T, K):
    """(rows per chunk, chunks) of mxm_coldot's partial buffer for a [T, K] operand."""
    return _query("mxm_coldot_chunks", T, K, n_out=2)


def glu_partition(T, N):
    """(column tiles per chunk, grid, xS_down partial slots) of mxm_gemm_glu."""
    return _query("mxm_gemm_glu_partition", T, N, n_out=3)


def mlp_fwd_partitions(T, N, R):
    return _query("mxm_mlp_fwd_partitions", T, N, R, n_out=1)[0]


def mlp_bwd_partitions(T, N, R):
    """(super block rows, dxa partial slots) of the backward epilogue."""
    return _query("mxm_mlp_bwd_partitions", T, N, R, n_out=2)
