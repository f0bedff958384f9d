"""CPU oracle for the MXFP8 quantizer and the fused SwiGLU-LoRA MLP.

TEST INFRASTRUCTURE ONLY. This module is the checker the CUDA path is compared
against, and the CPU baseline that ``bench.py --impl reference`` times.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it; the product modules (``mxfp8``, ``fused_mlp``) never do.

It is a numpy restatement of the reference algorithm, with the same rounding
points.  Every function cites the reference line it follows (paths relative to
the reference project root):

* quantizer            -- scripts/mxfp8.py:46-86 (``_quant_kernel``, ``mx_quant``)
* blocked scale layout -- scripts/mxfp8.py:69-75, scripts/fused_mlp.py:59-62
* weight quantizer     -- scripts/mxfp8.py:40-43 (``quant_ref``; torchao 0.18.0
                          ``to_mx(..., RCEIL)`` + ``to_blocked``, which the
                          reference states is identical to ``mx_quant``,
                          scripts/mxfp8.py:11)
* MXFP8 GEMM           -- ``torch._scaled_mm`` at scripts/fused_mlp.py:279,283,
                          309,329: dequantize both operands, fp32 matmul, bf16 out
* MLP forward          -- scripts/fused_mlp.py:263-293 with the epilogue of
                          scripts/fused_mlp.py:65-109,198-215
* MLP backward         -- scripts/fused_mlp.py:295-336 with the epilogue of
                          scripts/fused_mlp.py:112-175,235-259

Parity is pinned by ``tests/golden/`` fixtures that were produced by running the
reference's own Triton quantizer and MLP code (see
``tests/golden/make_golden.py``) and by known-answer vectors.

Conventions: bf16 tensors are carried as float32 arrays whose values are
exactly representable in bf16; codes and scales are uint8 arrays.
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0


# --------------------------------------------------------------------------- scalar formats
def bf16_round(x):
    """Round float32 to the nearest bf16 (ties to even); NaN stays NaN, inf stays inf.

    This is every ``.to(torch.bfloat16)`` / ``.to(tl.bfloat16)`` in the reference.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32)
    bias = np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))
    r = ((b + bias) & np.uint32(0xFFFF0000)).view(np.float32)
    return np.where(np.isnan(x), np.float32(np.nan), r).astype(np.float32)


def bf16_bits_to_f32(u16):
    """bf16 bit patterns (uint16) -> float32 values (exact)."""
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(x):
    """float32 values (already bf16-representable) -> uint16 bit patterns."""
    return (np.ascontiguousarray(bf16_round(x)).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def e8m0_rceil(descale):
    """``cvt.rp.satfinite.ue8m0x2.f32`` restated from float32 bits (scripts/mxfp8.py:62-63).

    Rounds the power-of-two scale UP (toward +inf): code = biased exponent, +1 if
    any mantissa bit is set.  NaN -> 255, +inf and anything above 2^127 -> 254
    (satfinite), 0 and values <= 2^-127 -> 0, (2^-127, 2^-126) -> 1.
    """
    d = np.ascontiguousarray(descale, dtype=np.float32)
    b = d.view(np.uint32)
    exp = ((b >> np.uint32(23)) & np.uint32(0xFF)).astype(np.int64)
    man = (b & np.uint32(0x7FFFFF)).astype(np.int64)
    code = exp + (man != 0)
    sub = exp == 0
    code = np.where(sub, np.where(man > (1 << 22), 1, 0), code)
    code = np.minimum(code, 254)
    code = np.where(np.isnan(d), 255, code)
    return code.astype(np.uint8)


def e8m0_reciprocal(e):
    """The multiplier applied before the e4m3 cast (scripts/mxfp8.py:64-65).

    255 -> NaN (the reference multiplies by the NaN descale), 254 -> 2^-127,
    0 -> 1.0, otherwise 2^(127-e).
    """
    e = np.asarray(e).astype(np.int64)
    p = np.ldexp(np.float64(1.0), 127 - e)
    r = np.where(e == 255, np.nan, np.where(e == 254, 2.0 ** -127, np.where(e == 0, 1.0, p)))
    return r.astype(np.float32)


def e4m3_encode(v):
    """float32 -> E4M3 (fn) code, round to nearest even, subnormals kept.

    Inputs are already clamped to [-448, 448] (scripts/mxfp8.py:66) or NaN.
    NaN -> 0x7F; the sign of zero is kept (-0 -> 0x80).
    """
    v = np.ascontiguousarray(v, dtype=np.float32)
    sign = ((v.view(np.uint32) >> np.uint32(31)) & np.uint32(1)).astype(np.uint8)
    a = np.abs(v.astype(np.float64))
    nan = np.isnan(a)
    a = np.where(nan, 0.0, a)
    # subnormal range: step 2^-9; RNE with np.rint (round half to even)
    sub_q = np.rint(a * 512.0)                       # 0..8 (8 == smallest normal, code 0x08)
    f, ex = np.frexp(a)                              # a = f * 2^ex, f in [0.5, 1)
    e = (ex - 1).astype(np.int64)
    e = np.where(a >= 2.0 ** -6, e, -6)
    # normal: mantissa steps of 2^(e-3); value/2^(e-3) in [8, 16)
    m = np.rint(a / np.ldexp(1.0, e - 3))
    carry = m >= 16
    e = np.where(carry, e + 1, e)
    m = np.where(carry, 8, m)
    normal_code = ((e + 7).astype(np.int64) << 3) | (m.astype(np.int64) - 8)
    code = np.where(a >= 2.0 ** -6, normal_code, sub_q.astype(np.int64))
    code = np.where(nan, 0x7F, code | (sign.astype(np.int64) << 7))
    return code.astype(np.uint8)


_E4M3_TABLE = None


def e4m3_decode(codes):
    """E4M3 (fn) code -> float32 value (0x7F / 0xFF -> NaN)."""
    global _E4M3_TABLE
    if _E4M3_TABLE is None:
        t = np.zeros(256, dtype=np.float32)
        for c in range(256):
            s = -1.0 if c & 0x80 else 1.0
            ex = (c >> 3) & 0xF
            mn = c & 7
            if ex == 0xF and mn == 7:
                t[c] = np.nan
            elif ex == 0:
                t[c] = s * mn * 2.0 ** -9
            else:
                t[c] = s * (1 + mn / 8.0) * 2.0 ** (ex - 7)
        _E4M3_TABLE = t
    return _E4M3_TABLE[np.asarray(codes, dtype=np.uint8)]


# --------------------------------------------------------------------------- blocked scale layout
def scale_bytes(rows, cols):
    """Size of the blocked scale buffer for a [rows, cols] operand (scripts/mxfp8.py:83-84)."""
    return -(-rows // 128) * (cols // 128) * 512


def scale_offsets(rows, cols):
    """Byte offset of the scale of (row r, 32-block kb) for every r < ceil128(rows), kb < cols/32.

    ((r // 128) * (cols / 128) + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
    (scripts/mxfp8.py:69,74; scripts/fused_mlp.py:59-61).
    """
    rp = -(-rows // 128) * 128
    r = np.arange(rp, dtype=np.int64)[:, None]
    kb = np.arange(cols // 32, dtype=np.int64)[None, :]
    return ((r // 128) * (cols // 128) + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4


def unblock_scales(s, rows, cols):
    """Blocked scale buffer -> [rows, cols/32] uint8 matrix."""
    off = scale_offsets(rows, cols)[:rows]
    return np.asarray(s, dtype=np.uint8)[off]


# --------------------------------------------------------------------------- quantizer
def mx_quant(x):
    """Row-wise MXFP8 quantization of a [R, K] bf16-valued array, K % 128 == 0.

    Follows ``_quant_kernel`` (scripts/mxfp8.py:46-75):
      amax over each 32-element block, NaN if the block has a NaN (:58-60);
      descale = amax / 448 in float32 (:61);  e = rceil_e8m0(descale) (:62-63);
      q = e4m3_rne(clamp(x * rcp(e), -448, 448)) (:64-67);
      scales in the blocked layout, padded rows (>= R) get scale 0 (:69-75).
    Returns (codes uint8 [R, K], scales uint8 flat [ceil(R/128) * K/128 * 512]).
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, K = x.shape
    assert K % 128 == 0, K
    xb = x.reshape(R, K // 32, 32)
    amax = np.max(np.abs(xb), axis=2).astype(np.float32)                  # np.max propagates NaN
    with np.errstate(invalid="ignore"):
        descale = (amax / np.float32(E4M3_MAX)).astype(np.float32)  # IEEE float32 division
    e = e8m0_rceil(descale)
    rcp = e8m0_reciprocal(e)
    with np.errstate(invalid="ignore", over="ignore"):
        q = (xb * rcp[:, :, None]).astype(np.float32)
        q = np.clip(q, -E4M3_MAX, E4M3_MAX)                          # NaN propagates (torch.clamp / torchao)
    codes = e4m3_encode(q).reshape(R, K)
    s = np.zeros(scale_bytes(R, K), dtype=np.uint8)
    off = scale_offsets(R, K)
    s[off[:R].ravel()] = e.ravel()
    return codes, s


def mx_quant_cols(x):
    """Column-wise quantization: the row-wise quantization of x^T (blocks of 32 along R).

    This is ``quant_ref(W.t().contiguous())`` (scripts/mxfp8.py:478,490).
    Returns (codes uint8 [K, R], scales for the [K, R] operand).
    """
    return mx_quant(np.ascontiguousarray(np.asarray(x, dtype=np.float32).T))


def mx_dequant(codes, s, rows, cols):
    """codes [rows, cols] + blocked scales -> float32 values code * 2^(e-127) (e=255 -> NaN)."""
    e = unblock_scales(s, rows, cols).astype(np.int64)
    mult = np.where(e == 255, np.nan, np.ldexp(1.0, e - 127)).astype(np.float64)
    v = e4m3_decode(codes).reshape(rows, cols // 32, 32).astype(np.float64) * mult[:, :, None]
    return v.reshape(rows, cols).astype(np.float32)


def mx_gemm(qa, sa, qb, sb, M, N, K):
    """``torch._scaled_mm(qa, qb.t(), sa, sb, out_dtype=bf16)``: D[M, N] = dq(A) @ dq(B)^T, fp32 sum, bf16 out.

    A is [M, K] and B is [N, K], both quantized along K.
    """
    a = mx_dequant(qa, sa, M, K)
    b = mx_dequant(qb, sb, N, K)
    return bf16_round(np.matmul(a, b.T, dtype=np.float32))


# --------------------------------------------------------------------------- weights (enable_mxfp8)
class MXWeights:
    """Frozen MLP weights in the layout ``enable_mxfp8`` builds (scripts/mxfp8.py:472-490).

    w_gu / ws_gu   : [W_gate; W_up] [2N, H] quantized along H (forward GEMM-1)
    wt_gu / wts_gu : [W_gate; W_up]^T [H, 2N] quantized along 2N (dx GEMM-4)
    w_d / ws_d     : W_down [H, N] quantized along N (forward GEMM-2)
    wt_d / wts_d   : W_down^T [N, H] quantized along H (dh GEMM-3)
    """

    def __init__(self, w_gate, w_up, w_down):
        w_gu = np.concatenate([np.asarray(w_gate, np.float32), np.asarray(w_up, np.float32)], 0)
        self.N, self.H = np.asarray(w_gate).shape
        self.w_gu, self.ws_gu = mx_quant(w_gu)
        self.wt_gu, self.wts_gu = mx_quant_cols(w_gu)
        self.w_d, self.ws_d = mx_quant(w_down)
        self.wt_d, self.wts_d = mx_quant_cols(w_down)


# --------------------------------------------------------------------------- fused MLP
def _silu_parts(g):
    """silu = g / (exp(-g) + 1) (scripts/fused_mlp.py:104,152) in float32."""
    with np.errstate(over="ignore"):
        return (g / (np.exp(-g) + np.float32(1.0))).astype(np.float32)


def _sigmoid(g):
    """tl.sigmoid = 1 / (1 + exp(-g)) (scripts/fused_mlp.py:158)."""
    with np.errstate(over="ignore"):
        return (np.float32(1.0) / (np.float32(1.0) + np.exp(-g))).astype(np.float32)


def _gu(gu, xs, bg, bu, s_g, s_u, N, r):
    """g, u = bf16(gu_half + s * xa @ B^T) (scripts/fused_mlp.py:65-71)."""
    g = bf16_round(gu[:, :N] + np.float32(s_g) * np.matmul(xs[:, :r], bg.T, dtype=np.float32))
    u = bf16_round(gu[:, N:] + np.float32(s_u) * np.matmul(xs[:, r:2 * r], bu.T, dtype=np.float32))
    return g, u


def fwd_epilogue(gu, xs, bg, bu, ad, s_g, s_u):
    """``mlp_fwd`` / ``_fwd_kernel`` (scripts/fused_mlp.py:65-109,198-215) on gu [T, 2N]: returns
    (h, q_h, s_h, xS_down) with h = bf16(silu(g) u), MXFP8(h) along N and xS_down = bf16(h Ad^T)."""
    N, r = gu.shape[1] // 2, ad.shape[0]
    g, u = _gu(gu, xs, bg, bu, s_g, s_u, N, r)                               # :69-70
    h = bf16_round(_silu_parts(g) * u)                                       # :104
    qh, sh = mx_quant(h)                                                     # :106 (_mx_store)
    xsd = bf16_round(np.matmul(h, ad.T, dtype=np.float32))                   # :108,214
    return h, qh, sh, xsd


def bwd_epilogue(gu, xs, dhm, dxd, bg, bu, ad, s_g, s_u):
    """``mlp_bwd`` / ``_bwd_kernel`` (scripts/fused_mlp.py:112-175,235-259) on gu [T, 2N] and dh_mx [T, N]:
    MXFP8([dg | du]) and the unscaled fp32 products dBg = dg^T xa_g, dBu = du^T xa_u, dAd = (h^T dxd)^T,
    dxa_g = dg Bg, dxa_u = du Bu, xS_down = h Ad^T."""
    N, r = gu.shape[1] // 2, ad.shape[0]
    g, u = _gu(gu, xs, bg, bu, s_g, s_u, N, r)                               # :151
    silu = _silu_parts(g)                                                    # :152
    h = bf16_round(silu * u)                                                 # :153
    dh = bf16_round(dhm + np.matmul(dxd, ad, dtype=np.float32))              # :155
    du = bf16_round(dh * silu)                                               # :157
    sig = _sigmoid(g)                                                        # :158
    dg = bf16_round(((dh * u) * sig) * (g * (np.float32(1.0) - sig) + np.float32(1.0)))   # :159
    dgu = np.concatenate([dg, du], 1)
    q_dgu, s_dgu = mx_quant(dgu)                                             # :160-162 (per-block == whole row)
    return dict(
        dg=dg, du=du, h=h, q_dgu=q_dgu, s_dgu=s_dgu,
        dBg=np.matmul(dg.T, xs[:, :r], dtype=np.float32),                    # :163
        dBu=np.matmul(du.T, xs[:, r:2 * r], dtype=np.float32),               # :164
        dAd=np.matmul(h.T, dxd, dtype=np.float32).T.copy(),                  # :165,175
        dxa_g=np.matmul(dg, bg, dtype=np.float32),                           # :166
        dxa_u=np.matmul(du, bu, dtype=np.float32),                           # :167
        xsd=np.matmul(h, ad.T, dtype=np.float32))                            # :168


def lora_params_bf16(Ag, Bg, Au, Bu, Ad, Bd):
    """The bf16 casts ``_MLP.forward`` makes of the LoRA parameters (scripts/fused_mlp.py:272-276)."""
    S = bf16_round(np.concatenate([Ag, Au], 0))
    return S, bf16_round(Bg), bf16_round(Bu), bf16_round(Ad), bf16_round(Bd)


def mlp_forward(x, W: MXWeights, Ag, Bg, Au, Bu, Ad, Bd, s_g, s_u, s_d, need_out=True):
    """``_MLP.forward`` (scripts/fused_mlp.py:263-293).

    x: [T, H] bf16 values.  Returns (y [T, H] or None, ctx dict of saved tensors).
    """
    x = np.asarray(x, np.float32)
    T, H = x.shape
    N, r = W.N, np.asarray(Ag).shape[0]
    S, bg, bu, ad, bd = lora_params_bf16(Ag, Bg, Au, Bu, Ad, Bd)
    xs = bf16_round(np.matmul(x, S.T, dtype=np.float32))                      # :277
    q, sc = mx_quant(x)                                                      # :278
    gu = mx_gemm(q, sc, W.w_gu, W.ws_gu, T, 2 * N, H)                        # :279
    ctx = dict(x=x, xs=xs, gu=gu, S=S, bg=bg, bu=bu, ad=ad, bd=bd, s=(s_g, s_u, s_d), W=W, r=r)
    if not need_out:
        return None, ctx
    h, qh, sh, xsd = fwd_epilogue(gu, xs, bg, bu, ad, s_g, s_u)
    y = mx_gemm(qh, sh, W.w_d, W.ws_d, T, H, N)                              # :283
    y = bf16_round(y + np.float32(s_d) * np.matmul(xsd, bd.T, dtype=np.float32))   # :284 addmm_
    ctx.update(h=h, qh=qh, sh=sh, xsd=xsd)
    return y, ctx


def mlp_backward(dy, ctx, need_x=True):
    """``_MLP.backward`` (scripts/fused_mlp.py:295-336) with the ``_bwd_kernel`` math (:112-175).

    Returns dict with dx [T, H] (bf16 values), dAg, dAu [r, H] (bf16 values),
    dBg, dBu [N, r] (fp32), dAd [r, N] (fp32), dBd [H, r] (bf16 values), and the
    intermediates q_dgu / s_dgu for byte-level checks.
    """
    W = ctx["W"]
    x, xs, gu, S, bg, bu, ad, bd = (ctx[k] for k in ("x", "xs", "gu", "S", "bg", "bu", "ad", "bd"))
    s_g, s_u, s_d = ctx["s"]
    r = ctx["r"]
    dy = bf16_round(np.asarray(dy, np.float32))
    T, H = dy.shape
    N = W.N
    qd, sd = mx_quant(dy)                                                    # :307
    dhm = mx_gemm(qd, sd, W.wt_d, W.wts_d, T, N, H)                          # :309
    dxd = bf16_round(np.matmul(dy, bd, dtype=np.float32))                    # :311
    if s_d != 1:
        dxd = bf16_round(dxd * np.float32(s_d))                              # :312-313
    e = bwd_epilogue(gu, xs, dhm, dxd, bg, bu, ad, s_g, s_u)                 # mlp_bwd / _bwd_kernel
    q_dgu, s_dgu, dBg, dBu, dAd = e["q_dgu"], e["s_dgu"], e["dBg"], e["dBu"], e["dAd"]
    dxa_g, dxa_u, xsd = e["dxa_g"], e["dxa_u"], e["xsd"]
    dBd = bf16_round(np.matmul(dy.T, bf16_round(xsd), dtype=np.float32))     # :316
    if s_d != 1:
        dBd = bf16_round(dBd * np.float32(s_d))                              # :317-318
    if s_g != 1:
        dxa_g = (dxa_g * np.float32(s_g)).astype(np.float32)                 # :320-322
        dBg = (dBg * np.float32(s_g)).astype(np.float32)
    if s_u != 1:
        dxa_u = (dxa_u * np.float32(s_u)).astype(np.float32)                 # :323-325
        dBu = (dBu * np.float32(s_u)).astype(np.float32)
    dxa = bf16_round(np.concatenate([dxa_g, dxa_u], 1))                      # :326
    out = dict(dBg=dBg, dBu=dBu, dAd=dAd, dBd=dBd, q_dgu=q_dgu, s_dgu=s_dgu, dhm=dhm, dxd=dxd, dxa=dxa)
    if need_x:
        dx = mx_gemm(q_dgu, s_dgu, W.wt_gu, W.wts_gu, T, H, 2 * N)           # :329
        dx = bf16_round(dx + np.matmul(dxa, S, dtype=np.float32))            # :331 addmm_
        out["dx"] = dx
    dA = bf16_round(np.matmul(dxa.T, x, dtype=np.float32))                   # :333
    out["dAg"], out["dAu"] = dA[:r], dA[r:]
    return out


def rel_fro(a, b):
    """Relative Frobenius error ||a - b|| / ||b|| (float64)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
