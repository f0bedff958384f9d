"""The allocation-free entry point mxm_coldot_noalloc against the regular mxm_coldot.

mxm_coldot_noalloc serves callers that cannot allocate device memory (code running inside a custom
device allocator, or services that reserve their whole memory budget up front): it keeps its partial
sums in one fixed device array instead of a caller-allocated buffer.  This file is collected last so a
stop-at-first-failure run has already run every other test; it passes alone and after the others.
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


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("T,K,n,post,tr", [(16384, 2048, 16, 2.0, False), (3000, 1024, 32, 1.0, True),
                                           (77, 6144, 64, 1.0, False)])
def test_noalloc_matches_coldot_twice(T, K, n, post, tr):
    import fused_mlp
    g = torch.Generator(device="cpu").manual_seed(T + K + n)
    for call in range(2):   # two calls in a row: the shared scratch keeps the previous call's partials
        A = torch.randn(T, K, generator=g).to(torch.bfloat16).cuda()
        E = (torch.randn(T, n, generator=g) * 0.1).to(torch.bfloat16).cuda()
        ref = fused_mlp.coldot(A, E, post=post, transpose_out=tr)
        out = _noalloc(A, E, post, transpose_out=tr)
        torch.cuda.synchronize()
        assert out.shape == ref.shape
        assert _rel(out.float(), ref.float()) < 5e-3, (call, _rel(out.float(), ref.float()))


def test_noalloc_rejects_oversized_request():
    import _mxlib
    A = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_mxlib.MXError) as ei:
        # K * n = 131072 * 64 exceeds the fixed scratch: rejected before any device access
        _mxlib.call("mxm_coldot_noalloc", _mxlib.ptr(A), 64, _mxlib.ptr(A), 64, 128, 131072, 64, 1.0, 0,
                    _mxlib.ptr(A), _mxlib.stream_of(A))
    assert "scratch" in str(ei.value)
