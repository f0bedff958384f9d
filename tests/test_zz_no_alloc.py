"""The allocation-free entry point mxm_coldot_noalloc.

mxm_coldot_noalloc serves callers that cannot allocate device memory (code running inside a custom
device allocator, or services that reserve their whole memory budget up front): it keeps its partial
sums in one fixed device array instead of a caller-allocated buffer.  It is checked against an fp32
torch reference of A^T E and, bit for bit, against the regular mxm_coldot with the same row chunking, on
two calls in a row (the shared array keeps the previous call's partials).  This file is collected last
so a stop-at-first-failure run has already run every other test; it passes alone and after the others.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(A, E, post, transpose_out=False):
    import _mxlib
    T, K = A.shape
    n = E.shape[1]
    out = torch.empty((n, K) if transpose_out else (K, n), dtype=torch.bfloat16, device=A.device)
    _mxlib.call("mxm_coldot_noalloc", _mxlib.ptr(A), A.stride(0), _mxlib.ptr(E), E.stride(0), T, K, n,
                float(post), 1 if transpose_out else 0, _mxlib.ptr(out), _mxlib.stream_of(A))
    return out


def _coldot_chunked(A, E, post, transpose_out, rpc, chunks):
    """mxm_coldot with an explicit row chunking (a caller-allocated partial buffer)."""
    import _mxlib
    T, K = A.shape
    n = E.shape[1]
    part = torch.empty((chunks, K, n), dtype=torch.float32, device=A.device)
    out = torch.empty((n, K) if transpose_out else (K, n), dtype=torch.bfloat16, device=A.device)
    _mxlib.call("mxm_coldot", _mxlib.ptr(A), A.stride(0), _mxlib.ptr(E), E.stride(0), T, K, n, float(post),
                1 if transpose_out else 0, _mxlib.ptr(part), rpc, chunks, _mxlib.ptr(out), 0, _mxlib.stream_of(A))
    return out


def _chunks(T, K, n, num_sms=0):
    import _mxlib
    rpc, nch = ctypes.c_int(0), ctypes.c_int(0)
    _mxlib.call("mxm_coldot_noalloc_chunks", T, K, n, num_sms, ctypes.byref(rpc), ctypes.byref(nch))
    return rpc.value, nch.value


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("T,K,n,post,tr", [(16384, 2048, 16, 2.0, False), (3000, 1024, 32, 1.0, True),
                                           (77, 6144, 64, 1.0, False)])
def test_noalloc_matches_fp32_and_coldot_twice(T, K, n, post, tr):
    g = torch.Generator(device="cpu").manual_seed(T + K + n)
    rpc, nch = _chunks(T, K, n)
    for call in range(2):   # two calls in a row: the shared scratch keeps the previous call's partials
        A = torch.randn(T, K, generator=g).to(torch.bfloat16).cuda()
        E = (torch.randn(T, n, generator=g) * 0.1).to(torch.bfloat16).cuda()
        ref = (A.float().t() @ E.float()).to(torch.bfloat16).float() * post   # bf16(bf16(A^T E) * post)
        ref = ref.to(torch.bfloat16)
        if tr:
            ref = ref.t()
        same = _coldot_chunked(A, E, post, tr, rpc, nch)
        out = _noalloc(A, E, post, transpose_out=tr)
        torch.cuda.synchronize()
        assert out.shape == ref.shape and out.dtype == torch.bfloat16
        assert _rel(out.float(), ref.float()) < 5e-3, (call, _rel(out.float(), ref.float()))
        assert torch.equal(out.view(torch.int16), same.view(torch.int16)), call   # same chunking: same bits


def test_taller_chunks_of_a_larger_device_compute_the_same_sums():
    """On a device with many more SMs the no-alloc chunking caps the chunk count so the partials fit the
    fixed scratch.  A B200 never needs the cap; here the capped chunking of a 1,024-SM device drives the
    regular mxm_coldot and must still give A^T E."""
    T, K, n = 20000, 2048, 64
    rpc, nch = _chunks(T, K, n, num_sms=1024)
    assert nch * K * n * 4 <= 16 << 20 and rpc * nch >= T and rpc % 64 == 0
    g = torch.Generator(device="cpu").manual_seed(1)
    A = torch.randn(T, K, generator=g).to(torch.bfloat16).cuda()
    E = (torch.randn(T, n, generator=g) * 0.1).to(torch.bfloat16).cuda()
    out = _coldot_chunked(A, E, 1.0, False, rpc, nch)
    ref = (A.float().t() @ E.float())
    assert _rel(out.float(), ref) < 5e-3


def test_noalloc_rejects_oversized_request():
    import _mxlib
    A = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_mxlib.MXError) as ei:
        # K * n = 131072 * 64 exceeds the fixed scratch: rejected before any device access
        _mxlib.call("mxm_coldot_noalloc", _mxlib.ptr(A), 64, _mxlib.ptr(A), 64, 128, 131072, 64, 1.0, 0,
                    _mxlib.ptr(A), _mxlib.stream_of(A))
    assert "scratch" in str(ei.value)
