"""Grouped LoRA linears on the GPU: mxfp8.lora_bwd, mxfp8.res_lora and fused_linear.group_linear /
residual_add (the reference's scripts/mxfp8.py:88-296 and scripts/fused_linear.py).

Bars: MX codes and scales byte-identical to mx_quant (which the golden fixtures pin); d(xa), dB and the
residual within the stated tolerances of an fp32 torch computation of the same op; grouped and
module-by-module layers within 5e-3 relative Frobenius error (1e-2 for the module-by-module dx) of an
fp32 reference built from the oracle's MXFP8 quantizers (dequantize, then fp32 matmul).
"""
import numpy as np
import pytest
import torch
from torch import nn

pytestmark = pytest.mark.gpu
TOL = 5e-3


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _blocks(s, rows, cols):
    """Blocked scale layout [ceil(rows/128), cols/128, 512] bytes."""
    return s.view(torch.uint8).view(-(-rows // 128), cols // 128, 512)


@pytest.mark.parametrize("T,N,r", [(77, 1024, 16), (1000, 2048, 16), (4096, 1024, 32), (300, 512, 64)])
def test_lora_bwd_quant_dxa_db(T, N, r):
    import mxfp8
    g = torch.Generator().manual_seed(T + N + r)
    dev = torch.device("cuda")
    dy = torch.randn(T, N, generator=g).to(torch.bfloat16).to(dev)
    xS = (torch.randn(T, 3 * r, generator=g) * 0.5).to(torch.bfloat16).to(dev)   # the branch is a column slice
    xa = xS[:, r:2 * r]
    B = (torch.randn(N, r, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    off_tiles = 2                                                                # codes at columns 256 ..
    width = off_tiles * 128 + N + 128
    q = torch.zeros((T, width), dtype=mxfp8.F8, device=dev)
    s = torch.zeros(mxfp8.scale_numel(T, width), dtype=torch.uint8, device=dev)
    dS = torch.zeros((T, 3 * r), dtype=torch.bfloat16, device=dev)
    dB = mxfp8.lora_bwd(dy, xa, B, 2.0, q=q, s=s, col_tile_off=off_tiles, dxa_out=dS[:, :r])
    q0, s0 = mxfp8.mx_quant(dy)
    torch.cuda.synchronize()
    c0 = off_tiles * 128
    assert torch.equal(q.view(torch.uint8)[:, c0:c0 + N], q0.view(torch.uint8))
    assert torch.equal(_blocks(s, T, width)[:, off_tiles:off_tiles + N // 128], _blocks(s0, T, N))
    assert int(q.view(torch.uint8)[:, :c0].abs().sum()) == 0                     # other columns untouched
    ref_dxa = (dy.float() @ B.float()) * 2.0
    assert _rel(dS[:, :r], ref_dxa) < 1e-2
    assert int(dS[:, r:].float().abs().sum()) == 0
    ref_db = (dy.float().t() @ xa.float()) * 2.0
    assert dB.dtype == torch.float32 and _rel(dB, ref_db) < 1e-5
    import _mxlib
    assert _mxlib.device_error() == 0


def test_lora_bwd_quant_only_and_unsupported_rank():
    import _mxlib
    import mxfp8
    dev = torch.device("cuda")
    T, N = 513, 768
    dy = torch.randn(T, N, device=dev).to(torch.bfloat16)
    q = torch.empty((T, N), dtype=mxfp8.F8, device=dev)
    s = torch.empty(mxfp8.scale_numel(T, N), dtype=torch.uint8, device=dev)
    assert mxfp8.lora_bwd(dy, q=q, s=s) is None
    q0, s0 = mxfp8.mx_quant(dy)
    assert torch.equal(q.view(torch.uint8), q0.view(torch.uint8))
    assert torch.equal(s.view(torch.uint8), s0.view(torch.uint8))
    # rank 8: not a rank the kernels take -- an explicit MXM_ERR_UNSUPPORTED, no silent library fallback
    xa = torch.randn(T, 8, device=dev).to(torch.bfloat16)
    B = torch.randn(N, 8, device=dev).to(torch.bfloat16)
    dxa = torch.empty((T, 8), dtype=torch.bfloat16, device=dev)
    assert not mxfp8.lora_bwd_ok(dy, xa, B)
    with pytest.raises(_mxlib.MXError) as ei:
        mxfp8.lora_bwd(dy, xa, B, 0.5, dxa_out=dxa)
    assert ei.value.status == mxfp8.MXM_ERR_UNSUPPORTED


@pytest.mark.parametrize("T", [77, 1000])
def test_group_lora_bwd_matches_per_branch(T):
    """One native call for a group's backward (three branches, the middle one without LoRA) gives the same
    bytes as one lora_bwd call per branch."""
    import mxfp8
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(T)
    Ns, r = (512, 256, 384), 16
    dys = [torch.randn(T, n, generator=g).to(torch.bfloat16).to(dev) for n in Ns]
    xS = (torch.randn(T, 2 * r, generator=g) * 0.5).to(torch.bfloat16).to(dev)
    Bs = [(torch.randn(n, r, generator=g) * 0.05).to(torch.bfloat16).to(dev) for n in Ns]
    W = sum(Ns)
    outs = []
    for native in (True, False):
        q = torch.zeros((T, W), dtype=mxfp8.F8, device=dev)
        s = torch.zeros(mxfp8.scale_numel(T, W), dtype=torch.uint8, device=dev)
        dS = torch.zeros((T, 2 * r), dtype=torch.bfloat16, device=dev)
        dB0 = torch.empty((Ns[0], r), dtype=torch.float32, device=dev)
        dB2 = torch.empty((Ns[2], r), dtype=torch.float32, device=dev)
        if native:
            mxfp8.group_lora_bwd(T, [(dys[0], xS[:, :r], Bs[0].t().contiguous(), 2.0, dS[:, :r], dB0),
                                     (dys[1], None, None, 0.0, None, None),
                                     (dys[2], xS[:, r:], Bs[2].t().contiguous(), 0.5, dS[:, r:], dB2)], q, s)
        else:
            dB0 = mxfp8.lora_bwd(dys[0], xS[:, :r], Bs[0], 2.0, q=q, s=s, col_tile_off=0, dxa_out=dS[:, :r])
            mxfp8.lora_bwd(dys[1], q=q, s=s, col_tile_off=Ns[0] // 128)
            dB2 = mxfp8.lora_bwd(dys[2], xS[:, r:], Bs[2], 0.5, q=q, s=s, col_tile_off=(Ns[0] + Ns[1]) // 128,
                                 dxa_out=dS[:, r:])
        outs.append((q.view(torch.uint8), s, dS, dB0, dB2))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    assert _rel(outs[0][3], dys[0].float().t() @ xS[:, :r].float() * 2.0) < 1e-5


@pytest.mark.parametrize("T,N,r", [(1, 128, 16), (333, 2048, 16), (4096, 1024, 32)])
def test_res_lora(T, N, r):
    import mxfp8
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(T * 7 + N)
    x = torch.randn(T, N, generator=g).to(torch.bfloat16).to(dev)
    y = torch.randn(T, N, generator=g).to(torch.bfloat16).to(dev)
    xS = torch.randn(T, 2 * r, generator=g).to(torch.bfloat16).to(dev)
    B = (torch.randn(N, r, generator=g) * 0.1).to(torch.bfloat16).to(dev)
    out = mxfp8.res_lora(x, y, xS[:, r:], B, 2.0)
    t = (y.float() + 2.0 * (xS[:, r:].float() @ B.float().t())).to(torch.bfloat16)
    ref = (x.float() + t.float()).to(torch.bfloat16)
    torch.cuda.synchronize()
    same = (out == ref).float().mean().item()
    assert same > 0.999, same          # the r products are summed in another order: rare 1-ulp flips of t
    # a flip of the intermediate t = bf16(y + s xa B^T) by one of its ulps, carried through x + t
    bound = (t.float().abs() + ref.float().abs()) * 2.0 ** -7 * 1.01 + 1e-30
    assert bool(((out.float() - ref.float()).abs() <= bound).all())


def test_res_lora_rejects_what_it_does_not_take():
    import _mxlib
    import mxfp8
    x = torch.randn(64, 256, device="cuda").to(torch.bfloat16)
    xa = torch.randn(64, 8, device="cuda").to(torch.bfloat16)
    B = torch.randn(256, 8, device="cuda").to(torch.bfloat16)
    with pytest.raises(_mxlib.MXError) as ei:
        mxfp8.res_lora(x, x, xa, B, 1.0)
    assert ei.value.status == mxfp8.MXM_ERR_UNSUPPORTED


# ------------------------------------------------------------------------------------------------ group_linear
class _LoRA(nn.Module):
    """The attributes of a PEFT LoRA Linear that fused_linear._part reads, and its forward."""

    def __init__(self, base, r, alpha):
        super().__init__()
        self.base_layer = base
        self.lora_A = nn.ModuleDict({"default": nn.Linear(base.in_features, r, bias=False)})
        self.lora_B = nn.ModuleDict({"default": nn.Linear(r, base.out_features, bias=False)})
        nn.init.normal_(self.lora_A["default"].weight, std=0.02)
        nn.init.normal_(self.lora_B["default"].weight, std=0.02)
        self.lora_dropout = nn.ModuleDict({"default": nn.Identity()})
        self.scaling = {"default": alpha / r}
        self.active_adapters = ["default"]
        self.use_dora = {"default": False}
        self.lora_variant = {}
        self.merged = False
        self.disable_adapters = False

    def forward(self, x):
        return self.base_layer(x) + self.scaling["default"] * self.lora_B["default"](self.lora_A["default"](x))


H, KV, R = 512, 256, 16


def _lin(i, o):
    m = nn.Linear(i, o, bias=False).requires_grad_(False)
    nn.init.normal_(m.weight, std=0.02)
    return m


class _Attn(nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj, self.k_proj, self.v_proj = _LoRA(_lin(H, H), R, 32), _LoRA(_lin(H, KV), R, 32), _LoRA(_lin(H, KV), R, 32)
        self.o_proj = _LoRA(_lin(H, H), R, 32)


class _Gdn(nn.Module):
    """A DeltaNet-shaped block: in_proj_qkv / in_proj_z with LoRA, in_proj_b / in_proj_a plain frozen
    16-output linears (thin: computed inside the group's skinny product), out_proj with LoRA."""

    def __init__(self):
        super().__init__()
        self.in_proj_qkv, self.in_proj_z = _LoRA(_lin(H, 768), R, 16), _LoRA(_lin(H, 512), R, 16)
        self.in_proj_b, self.in_proj_a = _lin(H, 16), _lin(H, 16)
        self.out_proj = _LoRA(_lin(512, H), R, 16)


class _Model(nn.Module):
    """model.layers.{0: self_attn, 1: linear_attn} -- the module names enable_mxfp8 looks for."""

    def __init__(self):
        super().__init__()
        self.model = nn.Module()
        self.model.layers = nn.ModuleList([nn.ModuleDict({"self_attn": _Attn()}), nn.ModuleDict({"linear_attn": _Gdn()})])


def _np(t):
    return t.detach().float().cpu().numpy()


def _mx_rows(a):
    """Dequantized row-wise MXFP8 of a bf16 matrix (the oracle's quantizer)."""
    from oracle import mx_oracle as O
    q, s = O.mx_quant(a)
    return O.mx_dequant(q, s, *a.shape)


def _mx_cols_t(w):
    """W^T quantized along N (the oracle's column quantizer), dequantized and transposed back: [N, K]."""
    from oracle import mx_oracle as O
    q, s = O.mx_quant_cols(w)
    return O.mx_dequant(q, s, w.shape[1], w.shape[0]).T


def _oracle_group(x, mods, dys, bf16_w):
    """fp32 reference of one group call from the oracle's quantizers: outputs, dx, (dA, dB) per LoRA branch.
    MX outputs: MXFP8(x) against the row-quantized W; backward: MXFP8(dy) against W^T quantized along N;
    LoRA terms in fp32 from bf16 operands; thin frozen linears in fp32."""
    from oracle import mx_oracle as O
    bf = O.bf16_round
    xq = _mx_rows(x)
    outs, dx, grads = [], np.zeros_like(x), []
    for m, dy in zip(mods, dys):
        base = getattr(m, "base_layer", m)
        w = bf16_w[id(base)]
        if m is base:                                    # thin plain linear (bf16 weight, fp32 math)
            outs.append(x @ w.T)
            dx += dy @ w
            continue
        A, B = bf(_np(m.lora_A["default"].weight)), bf(_np(m.lora_B["default"].weight))
        s = m.scaling["default"]
        xa = bf(x @ A.T)
        outs.append(xq @ _mx_rows(w).T + s * (xa @ B.T))
        dyb = bf(dy)
        dxa = bf(s * (dyb @ B))
        dx += _mx_rows(dyb) @ _mx_cols_t(w) + dxa @ A
        grads += [dxa.T @ x, s * (dyb.T @ xa)]
    return outs, dx, grads


def _group_call(mods, x, dys, need_out=True):
    import fused_linear
    fused_linear.new_step()
    xin = x.clone().requires_grad_(True)
    outs = fused_linear.group_linear(xin, mods, need_out=need_out)
    sum((y.float() * d).sum() for y, d in zip(outs, dys)).backward()
    ps = [w for m in mods if hasattr(m, "lora_A") for w in (m.lora_A["default"].weight, m.lora_B["default"].weight)]
    grads = [p.grad.detach().clone() for p in ps]
    for p in ps:
        p.grad = None
    return [y.detach() for y in outs], xin.grad.detach(), grads


@pytest.mark.parametrize("T", [700, 2049])
def test_group_linear_vs_oracle(T):
    """q|k|v (LoRA width 48: torch LoRA products) and qkv|z|b|a (LoRA 32 + thin 32 = 64: every product on
    the kernels) through group_linear after enable_mxfp8, against the oracle-built fp32 reference: outputs,
    dx and every LoRA gradient within 5e-3.  Both groups take the one-read backward; need_out=False gives the
    same gradients."""
    import fused_linear
    import mxfp8
    from oracle import mx_oracle as O
    torch.manual_seed(T)
    model = _Model().cuda()
    attn, gdn = model.model.layers[0]["self_attn"], model.model.layers[1]["linear_attn"]
    groups = ((attn.q_proj, attn.k_proj, attn.v_proj), (gdn.in_proj_qkv, gdn.in_proj_z, gdn.in_proj_b, gdn.in_proj_a))
    bf16_w = {id(getattr(m, "base_layer", m)): O.bf16_round(_np(getattr(m, "base_layer", m).weight))
              for grp in groups for m in grp}
    for grp in groups:   # the plain thin linears stay bf16 on the device (enable_mxfp8 does not convert them)
        for m in grp:
            if not hasattr(m, "base_layer"):
                m.weight.data = m.weight.data.to(torch.bfloat16)
    assert mxfp8.enable_mxfp8(model) == 7      # q, k, v, o, in_proj_qkv, in_proj_z, out_proj
    try:
        g = torch.Generator(device="cuda").manual_seed(1)
        x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
        for grp in groups:
            dys = [torch.randn(T, getattr(m, "base_layer", m).out_features, device="cuda", generator=g)
                   .to(torch.bfloat16) for m in grp]
            n0 = fused_linear.STATS.get("lan ngược gộp", 0)
            outs, dx, grads = _group_call(grp, x, dys)
            assert fused_linear.STATS.get("lan ngược gộp", 0) == n0 + 1
            ro, rdx, rgr = _oracle_group(_np(x), grp, [_np(d) for d in dys], bf16_w)
            for a, b in zip(outs, ro):
                assert O.rel_fro(_np(a), b) < TOL
            assert O.rel_fro(_np(dx), rdx) < TOL
            for a, b in zip(grads, rgr):
                assert O.rel_fro(_np(a), b) < TOL
            _, dx2, grads2 = _group_call(grp, x, dys, need_out=False)
            assert torch.equal(dx, dx2) and all(torch.equal(a, b) for a, b in zip(grads, grads2))
    finally:
        mxfp8.disable_mxfp8(model)
    import _mxlib
    assert _mxlib.device_error() == 0


def test_module_calls_and_deferred_residual_vs_oracle():
    """The same linears called one by one through the patched forwards (the MX linear autograd node and its
    input-quantization reuse) and o_proj deferred into residual_add: outputs and gradients against the
    oracle-built reference."""
    import fused_linear
    import mxfp8
    from oracle import mx_oracle as O
    torch.manual_seed(5)
    model = _Model().cuda()
    attn = model.model.layers[0]["self_attn"]
    mods = (attn.q_proj, attn.k_proj, attn.v_proj)
    bf16_w = {id(m.base_layer): O.bf16_round(_np(m.base_layer.weight)) for m in mods + (attn.o_proj,)}
    mxfp8.enable_mxfp8(model)
    try:
        T = 333
        g = torch.Generator(device="cuda").manual_seed(2)
        x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
        dys = [torch.randn(T, m.base_layer.out_features, device="cuda", generator=g).to(torch.bfloat16) for m in mods]
        q0, u0 = mxfp8.STATS["quant"], mxfp8.STATS["reuse"]
        xin = x.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            outs = [m(xin) for m in mods]
        assert mxfp8.STATS["reuse"] - u0 == 2 and mxfp8.STATS["quant"] - q0 == 1   # q/k/v: one quantization
        sum((y.float() * d.float()).sum() for y, d in zip(outs, dys)).backward()
        ro, rdx, rgr = _oracle_group(_np(x), mods, [_np(d) for d in dys], bf16_w)
        for a, b in zip(outs, ro):
            assert O.rel_fro(_np(a), b) < TOL
        # dx: autograd adds the modules' bf16 gradients one by one (each rounded to bf16), hence 1e-2
        assert O.rel_fro(_np(xin.grad), rdx) < 1e-2
        # o_proj deferred: residual_add adds its LoRA term inside the residual kernel
        fused_linear.new_step()
        h = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
        r0 = fused_linear.STATS.get("residual LoRA", 0)
        (o,) = fused_linear.group_linear(h, (attn.o_proj,), defer=True)
        assert isinstance(o, fused_linear.Deferred)
        res = fused_linear.residual_add(x, o)
        assert fused_linear.STATS.get("residual LoRA", 0) == r0 + 1
        (ro_o,), _, _ = _oracle_group(_np(h), (attn.o_proj,), [np.zeros((T, H), np.float32)], bf16_w)
        assert O.rel_fro(_np(res), _np(x) + ro_o) < TOL
    finally:
        mxfp8.disable_mxfp8(model)
