"""Generate the golden fixtures in this directory from the REFERENCE implementation.

Run once, in a container that has the reference checkout (default path given by
``--ref``); the fixtures it writes are committed and the tests read only them.

What runs is the reference's own code, on the CPU:

* ``mxfp8.mx_quant`` (scripts/mxfp8.py:46-86) -- the Triton ``_quant_kernel``
  executed by Triton's CPU interpreter (``TRITON_INTERPRET=1``);
* ``fused_mlp.mlp_fwd`` / ``mlp_bwd`` (scripts/fused_mlp.py:198-259) -- the Triton
  ``_fwd_kernel`` / ``_bwd_kernel`` under the same interpreter;
* ``fused_mlp._MLP.forward`` / ``backward`` (scripts/fused_mlp.py:262-336) -- the
  reference's autograd Function, driving the two above.

Substitutions, each needed because the CPU cannot run the original piece:

1. the one inline PTX instruction ``cvt.rp.satfinite.ue8m0x2.f32``
   (scripts/mxfp8.py:62) is evaluated per its PTX ISA definition (round toward
   +inf to a power of two, saturate finite, NaN -> 0xFF);
2. the interpreter's own float conversions are replaced where they differ from
   the GPU: fp32 -> bf16 and fp32 -> fp8e4m3 use torch's CPU casts (round to
   nearest even), bf16 ``tl.dot`` operands are widened to fp32 before the
   matmul, and ``libdevice.exp`` is numpy's float32 exp;
3. ``torch._scaled_mm`` (cuBLASLt MXFP8, GPU only) is replaced by
   dequantize-both-operands + fp32 matmul + bf16 cast, the parity definition;
4. ``quant_ref`` needs torchao 0.18.0 (absent); the reference states it is
   identical to ``mx_quant`` (scripts/mxfp8.py:11), so weights are quantized with
   ``mx_quant`` on the (transposed) weight.

Usage:  python tests/golden/make_golden.py [--ref PATH_TO_REFERENCE]
"""
import argparse
import math
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


# ----------------------------------------------------------------------------- interpreter patches
def _ue8m0_rp_satfinite(d):
    """PTX cvt.rp.satfinite.ue8m0: smallest power of two >= d, as a biased exponent code."""
    out = np.empty(d.shape, dtype=np.uint16)
    flat = d.reshape(-1).astype(np.float64)
    res = out.reshape(-1)
    for i, v in enumerate(flat):
        if math.isnan(v):
            res[i] = 255
        elif v <= 0.0:
            res[i] = 0
        elif math.isinf(v):
            res[i] = 254
        else:
            m, ex = math.frexp(v)          # v = m * 2^ex, m in [0.5, 1)
            lg = ex - 1 if m == 0.5 else ex
            res[i] = min(max(lg + 127, 0), 254)
    return out


def _patch_interpreter():
    from triton.runtime import interpreter as I
    import triton.language as tl

    B = I.InterpreterBuilder

    def create_inline_asm(self, inlineAsm, constraints, values, type, isPure, pack):
        assert "cvt.rp.satfinite.ue8m0x2.f32" in inlineAsm, inlineAsm
        d = values[0].data.astype(np.float32)
        h = I.TensorHandle(_ue8m0_rp_satfinite(d), tl.uint16)
        return types.SimpleNamespace(get_result=lambda i: h)

    def _to_f32(h):
        if h.dtype.scalar == tl.bfloat16:
            return (h.data.astype(np.uint32) << np.uint32(16)).view(np.float32)
        return h.data.astype(np.float32)

    def _f32_to_bf16_bits(a):
        t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)
        return t.view(torch.int16).numpy().view(np.uint16)

    orig_cast = B.cast_impl

    def cast_impl(self, src, dst_type):
        s, d = src.dtype.scalar, dst_type.scalar
        if s == tl.float32 and d == tl.bfloat16:
            return I.TensorHandle(_f32_to_bf16_bits(src.data), d)
        if s == tl.bfloat16 and d == tl.float32:
            return I.TensorHandle(_to_f32(src), d)
        return orig_cast(self, src, dst_type)

    orig_fp_to_fp = B.create_fp_to_fp

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        d = dst_type.scalar
        if d == tl.float8e4nv:
            t = torch.from_numpy(_to_f32(src)).to(torch.float8_e4m3fn)
            return I.TensorHandle(t.view(torch.uint8).numpy(), d)
        if d == tl.bfloat16 and src.dtype.scalar == tl.float32:
            return I.TensorHandle(_f32_to_bf16_bits(src.data), d)
        return orig_fp_to_fp(self, src, dst_type, rounding_mode)

    orig_dot = B.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
            out = np.matmul(_to_f32(a), _to_f32(b), dtype=np.float32) + d.data.astype(np.float32)
            return I.TensorHandle(out.astype(np.float32), d.dtype.scalar)
        return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    def create_extern_elementwise(self, libName, libPath, symbol, argList, retType, isPure):
        assert "exp" in symbol and "exp2" not in symbol, symbol
        x = argList[0].data.astype(np.float32)
        with np.errstate(over="ignore"):
            return I.TensorHandle(np.exp(x).astype(np.float32), tl.float32)

    B.create_inline_asm = create_inline_asm
    B.cast_impl = cast_impl
    B.create_fp_to_bf16 = None
    B.create_fp_to_fp = create_fp_to_fp
    B.create_fp_trunc = cast_impl
    B.create_fp_ext = cast_impl
    B.create_dot = create_dot
    B.create_extern_elementwise = create_extern_elementwise


import triton  # noqa: E402
import triton.language as tl  # noqa: E402


@triton.jit
def _exp_f32(x):
    return tl.exp(x)


def _import_reference(ref):
    for name in ["torchao", "torchao.prototype", "torchao.prototype.mx_formats",
                 "torchao.prototype.mx_formats.config", "torchao.prototype.mx_formats.mx_tensor",
                 "torchao.prototype.mx_formats.utils"]:
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["torchao.prototype.mx_formats.config"].ScaleCalculationMode = types.SimpleNamespace(RCEIL=None)
    sys.modules["torchao.prototype.mx_formats.mx_tensor"].to_mx = None
    sys.modules["torchao.prototype.mx_formats.utils"].to_blocked = None
    sys.path.insert(0, os.path.join(ref, "scripts"))
    _patch_interpreter()
    import mxfp8
    import fused_mlp
    fused_mlp._SMS[0] = 148          # B200 SM count: only changes the fp32 partial-sum grouping
    # libdevice.exp is an extern stub the interpreter cannot call: float32 exp instead
    fused_mlp.libdevice = types.SimpleNamespace(exp=_exp_f32)
    return mxfp8, fused_mlp


# ----------------------------------------------------------------------------- _scaled_mm stand-in
def _unblock(s_u8, rows, cols):
    nkb = cols // 32
    r = torch.arange(rows)[:, None]
    kb = torch.arange(nkb)[None, :]
    off = ((r // 128) * (cols // 128) + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
    return s_u8.view(torch.uint8).reshape(-1)[off]


def _dequant(q, s, rows, cols):
    e = _unblock(s, rows, cols).to(torch.float64)
    mult = torch.where(e == 255, torch.full_like(e, float("nan")), torch.exp2(e - 127))
    v = q.view(torch.float8_e4m3fn).to(torch.float64).reshape(rows, cols // 32, 32) * mult[:, :, None]
    return v.reshape(rows, cols).to(torch.float32)


def _scaled_mm_cpu(a, b, scale_a, scale_b, out_dtype=torch.bfloat16, **kw):
    M, K = a.shape
    N = b.shape[1]
    A = _dequant(a.contiguous(), scale_a, M, K)
    Bt = _dequant(b.t().contiguous(), scale_b, N, K)
    return (A @ Bt.t()).to(out_dtype)


# ----------------------------------------------------------------------------- fixtures
def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def quant_fixtures(mxfp8):
    cases = {}
    # (1) every bf16 bit pattern, 32 consecutive patterns per block
    allp = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).reshape(512, 128)
    cases["allbits"] = allp
    # (2) edge blocks: amax = 7*2^k (exact power-of-two descale), +-1 ulp, zeros, -0, tiny, inf, huge
    rows = []
    for k in range(-133, 128, 3):
        for delta in (-1, 0, 1):
            a = torch.tensor(7.0 * 2.0 ** k if abs(k) < 127 else 7.0 * 2.0 ** max(min(k, 124), -130))
            a = a.to(torch.bfloat16)
            ab = a.view(torch.int16) + delta
            amax = ab.view(torch.bfloat16).float()
            blk = torch.linspace(-1, 1, 32) * amax
            blk[5] = amax
            rows.append(blk)
    rows.append(torch.zeros(32))
    rows.append(-torch.zeros(32))
    rows.append(torch.full((32,), 1e-40))
    rows.append(torch.full((32,), -3e-39))
    t = torch.randn(32); t[3] = float("inf"); rows.append(t)
    t = torch.randn(32); t[7] = -float("inf"); rows.append(t)
    t = torch.randn(32); t[0] = float("nan"); rows.append(t)
    rows.append(torch.full((32,), 3.0e38))
    rows.append(torch.full((32,), 448.0))
    rows.append(torch.full((32,), 449.0))
    n = len(rows)
    pad = (-n) % 4
    rows += [torch.randn(32)] * pad
    edge = torch.stack(rows).reshape(-1, 128).to(torch.bfloat16)
    cases["edge"] = edge
    # (3) N(0,1) with 0.5% x200 outliers and 0.1% exact zeros, ragged rows
    g = torch.Generator().manual_seed(1234)
    for R, K in ((77, 256), (200, 384), (1, 128), (129, 128), (256, 384)):
        x = torch.randn(R, K, generator=g)
        m = torch.rand(R, K, generator=g)
        x = torch.where(m < 0.005, x * 200, x)
        x = torch.where((m >= 0.005) & (m < 0.006), torch.zeros_like(x), x)
        cases[f"rand_{R}x{K}"] = x.to(torch.bfloat16)
    out = {}
    for name, x in cases.items():
        q, s = mxfp8.mx_quant(x.contiguous())
        out[f"{name}_x"] = _bits(x)
        out[f"{name}_q"] = q.view(torch.uint8).numpy()
        out[f"{name}_s"] = s.view(torch.uint8).numpy()
        if x.shape[0] % 128 == 0:
            qt, st = mxfp8.mx_quant(x.t().contiguous())     # column-wise (quant_ref of W^T)
            out[f"{name}_qt"] = qt.view(torch.uint8).numpy()
            out[f"{name}_st"] = st.view(torch.uint8).numpy()
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **out)
    print("quant fixtures:", sorted(cases))


def mlp_fixtures(mxfp8, fused_mlp):
    torch._scaled_mm = _scaled_mm_cpu
    T, H, N, r, alpha = 200, 256, 256, 16, 32
    s = alpha / r
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, H, generator=g)
    x = torch.where(torch.rand(T, H, generator=g) < 0.01, x * 100, x).to(torch.bfloat16)
    Wg = (torch.randn(N, H, generator=g) * 0.02).to(torch.bfloat16)
    Wu = (torch.randn(N, H, generator=g) * 0.02).to(torch.bfloat16)
    Wd = (torch.randn(H, N, generator=g) * 0.02).to(torch.bfloat16)
    Ag = torch.randn(r, H, generator=g) * 0.01
    Au = torch.randn(r, H, generator=g) * 0.01
    Ad = torch.randn(r, N, generator=g) * 0.01
    Bg = torch.randn(N, r, generator=g) * 0.01
    Bu = torch.randn(N, r, generator=g) * 0.01
    Bd = torch.randn(H, r, generator=g) * 0.01
    dy = torch.randn(T, H, generator=g).to(torch.bfloat16)

    # enable_mxfp8's layout (scripts/mxfp8.py:472-490), quant_ref -> mx_quant
    w = torch.cat([Wg, Wu]).contiguous()
    hold = types.SimpleNamespace(n=N, half_t=[None, None])
    hold.w, hold.ws = mxfp8.mx_quant(w)
    hold.wt, hold.wts = mxfp8.mx_quant(w.t().contiguous())
    down = types.SimpleNamespace(out_features=H)
    down._mx_w, down._mx_ws = mxfp8.mx_quant(Wd.contiguous())
    down._mx_wt, down._mx_wts = mxfp8.mx_quant(Wd.t().contiguous())

    params = [p.clone().requires_grad_(True) for p in (Ag, Bg, Au, Bu, Ad, Bd)]
    xr = x.clone().requires_grad_(True)
    y = fused_mlp._MLP.apply(xr, (hold, down, (s, s, s), torch.bfloat16), True, *params)
    y.backward(dy)
    # the epilogue kernels' byte outputs, for byte-level checks
    import fused_linear
    fused_linear.new_step()
    S = torch.cat([Ag, Au]).to(torch.bfloat16)
    xs = x @ S.t()
    q, sc = mxfp8.mx_quant(x)
    gu = torch._scaled_mm(q, hold.w.t(), sc, hold.ws, out_dtype=torch.bfloat16)
    bg, bu, ad = Bg.to(torch.bfloat16), Bu.to(torch.bfloat16), Ad.to(torch.bfloat16)
    qh, sh, xsd = fused_mlp.mlp_fwd(gu, xs, bg, bu, ad, s, s, True)
    out = dict(
        T=T, H=H, N=N, r=r, alpha=alpha,
        x=_bits(x), Wg=_bits(Wg), Wu=_bits(Wu), Wd=_bits(Wd), dy=_bits(dy),
        Ag=Ag.numpy(), Au=Au.numpy(), Ad=Ad.numpy(), Bg=Bg.numpy(), Bu=Bu.numpy(), Bd=Bd.numpy(),
        y=_bits(y.detach()), dx=_bits(xr.grad),
        dAg=params[0].grad.numpy(), dBg=params[1].grad.numpy(), dAu=params[2].grad.numpy(),
        dBu=params[3].grad.numpy(), dAd=params[4].grad.numpy(), dBd=params[5].grad.numpy(),
        gu=_bits(gu), xs=_bits(xs), q_h=qh.view(torch.uint8).numpy(), s_h=sh.view(torch.uint8).numpy(),
        xsd=_bits(xsd),
        w_gu_q=hold.w.view(torch.uint8).numpy(), w_gu_s=hold.ws.view(torch.uint8).numpy(),
        wt_gu_q=hold.wt.view(torch.uint8).numpy(), wt_gu_s=hold.wts.view(torch.uint8).numpy(),
    )
    np.savez_compressed(os.path.join(HERE, "mlp_golden.npz"), **out)
    print("mlp fixtures: y", tuple(y.shape), "dx", tuple(xr.grad.shape))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MX_REFERENCE_ROOT"),
                    help="root of the reference checkout (or set MX_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("--ref (or MX_REFERENCE_ROOT) is required")
    mxfp8, fused_mlp = _import_reference(args.ref)
    quant_fixtures(mxfp8)
    mlp_fixtures(mxfp8, fused_mlp)


if __name__ == "__main__":
    main()
