"""The CPU oracle against the golden fixtures made from the reference's own code.

These tests pin the oracle: the quantizer must match the reference's Triton
``_quant_kernel`` (scripts/mxfp8.py:46-86) byte for byte on every fixture, and
the MLP restatement must match the reference ``_MLP`` (scripts/fused_mlp.py:262-336)
within the tolerances below.
"""
import os

import numpy as np
import pytest

from oracle import mx_oracle as O

G = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def qg():
    return np.load(os.path.join(G, "quant_golden.npz"))


@pytest.fixture(scope="module")
def mg():
    return np.load(os.path.join(G, "mlp_golden.npz"))


def codes_equal(a, b):
    """Byte equality of E4M3 codes, where any two NaN codes (0x7F / 0xFF) count as equal.

    A NaN block quantizes to NaN codes; the sign bit of a NaN is not defined by
    the reference (a CPU keeps the operand's sign, the GPU returns a canonical NaN).
    """
    a = np.asarray(a, np.uint8)
    b = np.asarray(b, np.uint8)
    nan = ((a & 0x7F) == 0x7F) & ((b & 0x7F) == 0x7F)
    return bool(np.all((a == b) | nan))


def _cases(z):
    return sorted({k[:-2] for k in z.files if k.endswith("_x")})


def test_quant_rows_bit_exact(qg):
    for name in _cases(qg):
        x = O.bf16_bits_to_f32(qg[f"{name}_x"])
        q, s = O.mx_quant(x)
        assert codes_equal(q, qg[f"{name}_q"]), name
        assert np.array_equal(s, qg[f"{name}_s"]), name


def test_quant_cols_bit_exact(qg):
    n = 0
    for name in _cases(qg):
        if f"{name}_qt" not in qg.files:
            continue
        x = O.bf16_bits_to_f32(qg[f"{name}_x"])
        q, s = O.mx_quant_cols(x)
        assert codes_equal(q, qg[f"{name}_qt"]), name
        assert np.array_equal(s, qg[f"{name}_st"]), name
        n += 1
    assert n >= 2


def _mlp_inputs(mg):
    f = lambda k: O.bf16_bits_to_f32(mg[k])  # noqa: E731
    W = O.MXWeights(f("Wg"), f("Wu"), f("Wd"))
    s = float(mg["alpha"]) / float(mg["r"])
    args = [mg[k] for k in ("Ag", "Bg", "Au", "Bu", "Ad", "Bd")]
    return f("x"), W, args, s, f("dy")


def test_weight_layout_matches(mg):
    x, W, args, s, dy = _mlp_inputs(mg)
    assert np.array_equal(W.w_gu, mg["w_gu_q"]) and np.array_equal(W.ws_gu, mg["w_gu_s"])
    assert np.array_equal(W.wt_gu, mg["wt_gu_q"]) and np.array_equal(W.wts_gu, mg["wt_gu_s"])


def test_mlp_forward_epilogue_bytes(mg):
    """h's fp8 codes and scales from the oracle vs the reference ``_fwd_kernel``."""
    x, W, args, s, dy = _mlp_inputs(mg)
    y, ctx = O.mlp_forward(x, W, *args, s, s, s)
    assert np.array_equal(O.f32_to_bf16_bits(ctx["xs"]), mg["xs"])
    assert np.array_equal(O.f32_to_bf16_bits(ctx["gu"]), mg["gu"])
    # numpy's float32 exp stands in for libdevice exp on both sides, so the codes agree exactly
    assert codes_equal(ctx["qh"], mg["q_h"])
    assert np.array_equal(ctx["sh"], mg["s_h"])
    assert O.rel_fro(ctx["xsd"], O.bf16_bits_to_f32(mg["xsd"])) < 1e-4


def test_mlp_forward_backward_matches_reference(mg):
    x, W, args, s, dy = _mlp_inputs(mg)
    y, ctx = O.mlp_forward(x, W, *args, s, s, s)
    g = O.mlp_backward(dy, ctx)
    tol = 1e-4       # only fp32 summation order differs from the reference
    assert O.rel_fro(y, O.bf16_bits_to_f32(mg["y"])) < tol
    assert O.rel_fro(g["dx"], O.bf16_bits_to_f32(mg["dx"])) < tol
    for k in ("dAg", "dBg", "dAu", "dBu", "dAd", "dBd"):
        assert O.rel_fro(g[k], mg[k]) < tol, k


def test_scale_from_amax_bits_equals_division():
    """The kernels compute the E8M0 scale from the abs-max's bf16 bits, ((bits + 0x1F) >> 7) - 8 clamped
    at 0, +inf -> 254, NaN -> 255, instead of rceil(amax / 448) (scripts/mxfp8.py:60-63): same code for
    every non-negative bf16 value."""
    bits = np.arange(0, 0x8000, dtype=np.uint32)
    m = (bits << 16).view(np.float32)
    with np.errstate(invalid="ignore"):
        ref = O.e8m0_rceil(m / np.float32(448.0)).astype(np.int64)
    e = np.maximum(((bits.astype(np.int64) + 0x1F) >> 7) - 8, 0)
    e = np.where(bits == 0x7F80, 254, np.where(bits > 0x7F80, 255, e))
    assert np.array_equal(e, ref)


def test_scale_rule_matches_the_reference_arithmetic_on_b200():
    """tests/golden/scale_rule_b200.npz (made by make_scale_rule_b200.py on a B200) holds, for every
    non-negative bf16 block abs-max, the scale code of the reference's GPU arithmetic: Triton's fp32
    division amax / 448 followed by cvt.rp.satfinite.ue8m0 (scripts/mxfp8.py:61-63).  That division is not
    IEEE-exact (one ulp high in about half the quotients) but it is exact where amax = 7 * 2^k, so every
    code equals the kernels' rule from the abs-max's bits and the oracle's IEEE division."""
    z = np.load(os.path.join(G, "scale_rule_b200.npz"))
    bits = z["amax_bits"].astype(np.int64)
    e = z["e"].astype(np.int64)
    assert len(bits) == 0x8000 and str(z["device"]).startswith("NVIDIA B200")
    rule = np.maximum(((bits + 0x1F) >> 7) - 8, 0)
    rule = np.where(bits == 0x7F80, 254, np.where(bits > 0x7F80, 255, rule))
    assert np.array_equal(rule, e)
    amax = (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)
    with np.errstate(invalid="ignore"):
        assert np.array_equal(O.e8m0_rceil(amax / np.float32(448.0)).astype(np.int64), e)
    exact = (bits & 0x7F) == 0x60      # amax = 7 * 2^k: the quotient is a power of two
    assert np.array_equal(z["descale_bits"][exact & (bits < 0x7F80)],
                          (amax / np.float32(448.0)).view(np.uint32)[exact & (bits < 0x7F80)])
