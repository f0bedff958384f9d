"""CUDA quantizer vs the CPU oracle and the reference golden vectors: bit-exact codes and scales."""
import os

import numpy as np
import pytest
import torch

from oracle import mx_oracle as O

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(__file__), "golden")


def _nan_eq(a, b):
    a = np.asarray(a, np.uint8)
    b = np.asarray(b, np.uint8)
    return bool(np.all((a == b) | (((a & 0x7F) == 0x7F) & ((b & 0x7F) == 0x7F))))


def _to_dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def _rand(R, K, seed, outliers=0.005, zeros=0.001):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(R, K, generator=g)
    m = torch.rand(R, K, generator=g)
    x = torch.where(m < outliers, x * 200, x)
    x = torch.where((m >= outliers) & (m < outliers + zeros), torch.zeros_like(x), x)
    return x.to(torch.bfloat16)


def test_rows_golden():
    import mxfp8
    z = np.load(os.path.join(G, "quant_golden.npz"))
    for name in sorted({k[:-2] for k in z.files if k.endswith("_x")}):
        x = _to_dev(z[f"{name}_x"])
        q, s = mxfp8.mx_quant(x)
        torch.cuda.synchronize()
        assert _nan_eq(q.view(torch.uint8).cpu().numpy(), z[f"{name}_q"]), name
        assert np.array_equal(s.view(torch.uint8).cpu().numpy(), z[f"{name}_s"]), name


def test_cols_and_both_golden():
    import mxfp8
    z = np.load(os.path.join(G, "quant_golden.npz"))
    n = 0
    for name in sorted({k[:-3] for k in z.files if k.endswith("_qt")}):
        x = _to_dev(z[f"{name}_x"])
        qt, st = mxfp8.mx_quant_t(x)
        q, s, qt2, st2 = mxfp8.mx_quant_pair(x)
        torch.cuda.synchronize()
        for a, b in ((qt, z[f"{name}_qt"]), (qt2, z[f"{name}_qt"]), (q, z[f"{name}_q"])):
            assert _nan_eq(a.view(torch.uint8).cpu().numpy(), b), name
        for a, b in ((st, z[f"{name}_st"]), (st2, z[f"{name}_st"]), (s, z[f"{name}_s"])):
            assert np.array_equal(a.view(torch.uint8).cpu().numpy(), b), name
        n += 1
    assert n >= 2


@pytest.mark.parametrize("R,K", [(1, 128), (77, 1024), (1000, 3584), (2049, 2048), (4096, 6144)])
def test_rows_random_vs_oracle(R, K):
    import mxfp8
    x = _rand(R, K, seed=R * 7 + K)
    q, s = mxfp8.mx_quant(x.cuda())
    qo, so = O.mx_quant(x.float().numpy())
    assert _nan_eq(q.view(torch.uint8).cpu().numpy(), qo)
    assert np.array_equal(s.view(torch.uint8).cpu().numpy(), so)


@pytest.mark.parametrize("R,K", [(128, 128), (4096, 1024), (2048, 3584)])
def test_cols_random_vs_oracle(R, K):
    import mxfp8
    x = _rand(R, K, seed=R + K)
    q, s, qt, st = mxfp8.mx_quant_pair(x.cuda())
    qo, so = O.mx_quant_cols(x.float().numpy())
    assert _nan_eq(qt.view(torch.uint8).cpu().numpy(), qo)
    assert np.array_equal(st.view(torch.uint8).cpu().numpy(), so)


def test_full_size_properties():
    """At the sweep's largest sizes: row-wise of x^T equals column-wise of x, and dequantized
    values stay within one E4M3 step of the input (size-independent properties)."""
    import mxfp8
    x = _rand(16384, 2048, seed=3).cuda()
    q, s, qt, st = mxfp8.mx_quant_pair(x)
    q2, s2 = mxfp8.mx_quant(x.t().contiguous())
    assert torch.equal(qt.view(torch.uint8), q2.view(torch.uint8))
    assert torch.equal(st.view(torch.uint8), s2.view(torch.uint8))
    # determinism
    q3, s3 = mxfp8.mx_quant(x)
    assert torch.equal(q.view(torch.uint8), q3.view(torch.uint8)) and torch.equal(s.view(torch.uint8), s3.view(torch.uint8))


@pytest.mark.parametrize("R,K", [(77, 256), (300, 1024)])
def test_fallback_kernel_on_unaligned_code_rows(R, K):
    """A code row stride that is not a multiple of 16 bytes (and a strided input) takes the per-tile
    fallback kernel instead of the TMA one; both must give mx_quant's bytes exactly."""
    import _mxlib
    import mxfp8
    x = _rand(R, K, seed=R + K).cuda()
    wide = torch.zeros(R, K + 8, dtype=torch.bfloat16, device="cuda")
    wide[:, :K] = x
    xs = wide[:, :K]                                     # row stride K + 8 elements
    ldq = K + 8                                          # not a multiple of 16 bytes
    q = torch.zeros(R, ldq, dtype=torch.uint8, device="cuda")
    s = torch.zeros(mxfp8.scale_numel(R, K), dtype=torch.uint8, device="cuda")
    _mxlib.call("mxm_quant_rows", _mxlib.ptr(xs), R, K, K + 8, _mxlib.ptr(q), ldq, _mxlib.ptr(s),
                _mxlib.stream_of(xs))
    q0, s0 = mxfp8.mx_quant(x)
    torch.cuda.synchronize()
    assert torch.equal(q[:, :K], q0.view(torch.uint8))
    assert int(q[:, K:].sum()) == 0
    assert torch.equal(s, s0.view(torch.uint8))
    assert _mxlib.device_error() == 0


def test_scales_match_the_reference_arithmetic_on_b200():
    """Every non-negative bf16 value as the abs-max of a 32-element block (the other 31 elements a smaller
    value of the same sign pattern), quantized by the kernel row-wise and column-wise: the scale codes equal
    those of the reference's GPU arithmetic recorded in scale_rule_b200.npz (Triton's fp32 amax / 448, then
    cvt.rp.satfinite.ue8m0; see make_scale_rule_b200.py)."""
    import os
    import mxfp8
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "scale_rule_b200.npz"))
    bits = z["amax_bits"].astype(np.int64)
    want = z["e"]
    n = len(bits)                                   # 32,768 blocks = 256 rows x 128 blocks of 32
    rows, cols = 256, 128 * 32
    blk = np.zeros((n, 32), dtype=np.uint16)
    blk[:, 0] = bits                                # the block's abs-max (NaN / inf included)
    blk[:, 1::2] = (bits >> 1)[:, None]             # smaller magnitudes elsewhere, half of them negative
    blk[:, 2::2] = ((bits >> 2) | 0x8000)[:, None]
    x = torch.from_numpy(blk.reshape(rows, cols).view(np.int16)).view(torch.bfloat16).cuda()
    q, s = mxfp8.mx_quant(x)
    from oracle import mx_oracle as O
    got = O.unblock_scales(s.view(torch.uint8).cpu().numpy(), rows, cols).reshape(-1)
    assert np.array_equal(got, want)
    qt, st = mxfp8.mx_quant_t(x.t().contiguous())   # the column-wise kernel on the transpose: same blocks
    got_t = O.unblock_scales(st.view(torch.uint8).cpu().numpy(), rows, cols).reshape(-1)
    assert np.array_equal(got_t, want)
