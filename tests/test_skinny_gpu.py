"""The rank-n skinny products on the GPU: rowdot (and its fused MXFP8 twin) and coldot.

rowdot_quant must give exactly mx_quant's codes and scales (and the golden vectors), and exactly
rowdot's product; both products are checked against an fp32 torch reference with the bf16 rounding
tolerance written below.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-2   # relative Frobenius error of a bf16-rounded fp32 product


def _nan_eq(a, b):
    a = np.asarray(a, np.uint8)
    b = np.asarray(b, np.uint8)
    return bool(np.all((a == b) | (((a & 0x7F) == 0x7F) & ((b & 0x7F) == 0x7F))))


def _rand(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_rowdot_quant_golden():
    import fused_mlp
    z = np.load(os.path.join(G, "quant_golden.npz"))
    n_cases = 0
    for name in sorted({k[:-2] for k in z.files if k.endswith("_x")}):
        bits = np.ascontiguousarray(z[f"{name}_x"])
        x = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
        B = _rand((16, x.shape[1]), seed=3).cuda()
        out, q, s = fused_mlp.rowdot_quant(x, B)
        torch.cuda.synchronize()
        assert _nan_eq(q.view(torch.uint8).cpu().numpy(), z[f"{name}_q"]), name
        assert np.array_equal(s.view(torch.uint8).cpu().numpy(), z[f"{name}_s"]), name
        n_cases += 1
    assert n_cases >= 2


@pytest.mark.parametrize("T,K,n", [(1, 128, 16), (77, 1152, 32), (1000, 2048, 16), (2049, 3584, 32),
                                   (512, 2048, 64), (4096, 2048, 32)])
def test_rowdot_quant_matches_quant_and_rowdot(T, K, n):
    import fused_mlp
    import mxfp8
    x = _rand((T, K), seed=T + K + n).cuda()
    B = _rand((n, K), seed=n, scale=0.05).cuda()
    post = 0.5 if n == 16 else 1.0
    out, q, s = fused_mlp.rowdot_quant(x, B, post=post)
    q0, s0 = mxfp8.mx_quant(x)
    out0 = fused_mlp.rowdot(x, B, post=post)
    torch.cuda.synchronize()
    assert torch.equal(q.view(torch.uint8), q0.view(torch.uint8))
    assert torch.equal(s.view(torch.uint8), s0.view(torch.uint8))
    assert torch.equal(out, out0)                                     # same kernel body, same order
    ref = ((x.float() @ B.float().t()).to(torch.bfloat16).float() * post)
    assert _rel(out, ref) < TOL


@pytest.mark.parametrize("T,K,n", [(1, 128, 16), (300, 2048, 16), (2049, 2048, 32), (8192, 1024, 64)])
def test_coldot_vs_torch(T, K, n):
    import fused_mlp
    A = _rand((T, K), seed=T * 3 + K).cuda()
    E = _rand((T, n), seed=n + 1, scale=0.1).cuda()
    ref = (A.float().t() @ E.float()).to(torch.bfloat16).float() * 0.5
    out = fused_mlp.coldot(A, E, post=0.5)
    outT = fused_mlp.coldot(A, E, post=0.5, transpose_out=True)
    torch.cuda.synchronize()
    assert _rel(out, ref) < TOL
    assert torch.equal(outT, out.t().contiguous())


def test_tma_path_from_a_fresh_thread():
    """A thread whose first CUDA call is one of ours (autograd's device thread runs the backward's
    rowdot_quant first) still gets the TMA kernels: the tensor-map encoder runs with the device context
    bound, leaves no error, and the result equals the main thread's."""
    import threading

    import _mxlib
    import fused_mlp
    A = _rand((1024, 2048), 31).cuda()
    B = _rand((16, 2048), 32, 0.05).cuda()
    # the outputs go back to torch's cache, so the thread's allocations need no CUDA call of their own
    ref = [t.clone() for t in fused_mlp.rowdot_quant(A, B, post=2.0)]
    torch.cuda.synchronize()
    got, err = {}, {}

    def run():
        try:
            got["r"] = fused_mlp.rowdot_quant(A, B, post=2.0)
            torch.cuda.synchronize()
            err["msg"] = _mxlib.last_error()   # per-thread message: set by any failed call in this thread
        except Exception as e:   # pragma: no cover - reported below
            err["exc"] = repr(e)

    t = threading.Thread(target=run)
    t.start()
    t.join()
    assert "exc" not in err, err
    assert err["msg"] == "", err["msg"]
    for a, b in zip(ref, got["r"]):
        assert torch.equal(a.view(torch.uint8) if a.dtype != torch.bfloat16 else a,
                           b.view(torch.uint8) if b.dtype != torch.bfloat16 else b)
