"""The give-up path of the kernels' bounded waits, made to run out on purpose without faulting the GPU.

Every mbarrier wait in the library gives up after a wall-time limit, records a code in the device-side
error flag and lets its kernel return (no __trap, no hang).  mxm_selftest_wait launches one CTA that
waits on an mbarrier nothing arrives on, with a 1 ms limit: the wait runs out, the host reads
MXM_ERR_DEVICE and code 9 through mxm_device_error, the flag clears, and the context stays usable.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports():
    import _mxlib
    import mxfp8
    from oracle import mx_oracle as O
    torch.cuda.init()
    assert _mxlib.device_error() == 0
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _mxlib.call("mxm_selftest_wait", 1_000_000, s)       # 1 ms limit
    code = ctypes.c_int(0)
    st = _mxlib._lib.mxm_device_error(ctypes.byref(code), 1)
    assert st == _mxlib.MXM_ERR_DEVICE and code.value == 9, (st, code.value)
    assert "self-test" in _mxlib.last_error()
    assert _mxlib.device_error() == 0                   # cleared
    # the context is intact: a quantizer call afterwards is bit-exact
    x = torch.randn(256, 512).to(torch.bfloat16)
    q, sc = mxfp8.mx_quant(x.cuda())
    qo, so = O.mx_quant(x.float().numpy())
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), qo)
    assert np.array_equal(sc.view(torch.uint8).cpu().numpy(), so)
    assert _mxlib.device_error() == 0


def test_selftest_rejects_unbounded_limits():
    import _mxlib
    with pytest.raises(_mxlib.MXError):
        _mxlib.call("mxm_selftest_wait", 0, None)
    with pytest.raises(_mxlib.MXError):
        _mxlib.call("mxm_selftest_wait", 10**9, None)
