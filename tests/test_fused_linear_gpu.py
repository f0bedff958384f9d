"""Grouped LoRA linears on the GPU: mxfp8.lora_bwd, mxfp8.res_lora and fused_linear.group_linear /
residual_add (the reference's scripts/mxfp8.py:88-296 and scripts/fused_linear.py).

Bars: MX codes and scales byte-identical to mx_quant (which the golden fixtures pin); d(xa), dB and the
residual within the stated tolerances of an fp32 torch computation of the same op; the grouped layer
within 5e-3 relative Frobenius error of calling the modules one by one.
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


def test_lora_bwd_quant_only_and_other_rank():
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
    # rank 8: the torch GEMM path, same contract
    xa = torch.randn(T, 8, device=dev).to(torch.bfloat16)
    B = torch.randn(N, 8, device=dev).to(torch.bfloat16)
    dxa = torch.empty((T, 8), dtype=torch.bfloat16, device=dev)
    dB = mxfp8.lora_bwd(dy, xa, B, 0.5, dxa_out=dxa)
    assert _rel(dxa, dy.float() @ B.float() * 0.5) < 1e-2
    assert _rel(dB, dy.float().t() @ xa.float() * 0.5) < 1e-5


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


class _Attn(nn.Module):
    def __init__(self, H, kv, r):
        super().__init__()
        mk = lambda i, o: nn.Linear(i, o, bias=False).requires_grad_(False)  # noqa: E731
        self.q_proj = _LoRA(mk(H, H), r, 2 * r)
        self.k_proj = _LoRA(mk(H, kv), r, 2 * r)
        self.v_proj = _LoRA(mk(H, kv), r, 2 * r)
        self.o_proj = _LoRA(mk(H, H), r, 2 * r)


class _Decoder(nn.Module):
    def __init__(self, H, kv, r):
        super().__init__()
        self.layers = nn.ModuleList([nn.ModuleDict({"self_attn": _Attn(H, kv, r)})])


class _Model(nn.Module):
    """model.layers.0.self_attn.{q,k,v,o}_proj, the module names enable_mxfp8 looks for."""

    def __init__(self, H, kv, r):
        super().__init__()
        self.model = _Decoder(H, kv, r)
        self.layers = self.model.layers


def _build(seed):
    torch.manual_seed(seed)
    m = _Model(512, 256, 16).cuda()
    for lin in (m.layers[0]["self_attn"].q_proj.base_layer, m.layers[0]["self_attn"].k_proj.base_layer,
                m.layers[0]["self_attn"].v_proj.base_layer, m.layers[0]["self_attn"].o_proj.base_layer):
        nn.init.normal_(lin.weight, std=0.02)
    return m


def _step(model, x, dys, dres, grouped):
    import fused_linear
    fused_linear.new_step()
    a = model.layers[0]["self_attn"]
    xin = x.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        mods = (a.q_proj, a.k_proj, a.v_proj)
        outs = fused_linear.group_linear(xin, mods) if grouped else tuple(m(xin) for m in mods)
        (o,) = fused_linear.group_linear(outs[0], (a.o_proj,), defer=grouped) if grouped else (a.o_proj(outs[0]),)
        res = fused_linear.residual_add(xin, o) if grouped else xin + o
    loss = sum((y.float() * d).sum() for y, d in zip(outs, dys)) + (res.float() * dres).sum()
    loss.backward()
    ps = [p for n, p in model.named_parameters() if p.requires_grad]
    grads = [p.grad.detach().clone() for p in ps]
    for p in ps:
        p.grad = None
    return [y.detach() for y in outs] + [res.detach()], xin.grad.detach(), grads


def test_group_linear_matches_module_calls():
    import fused_linear
    import mxfp8
    model = _build(0)
    assert mxfp8.enable_mxfp8(model) == 4
    T = 700
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(T, 512, device="cuda", generator=g).to(torch.bfloat16)
    dys = [torch.randn(T, n, device="cuda", generator=g) for n in (512, 256, 256)]
    dres = torch.randn(T, 512, device="cuda", generator=g)
    n0 = fused_linear.STATS.get("lan ngược gộp", 0)
    r0 = fused_linear.STATS.get("residual LoRA", 0)
    outs_g, dx_g, gr_g = _step(model, x, dys, dres, True)
    assert fused_linear.STATS.get("lan ngược gộp", 0) == n0 + 2      # both groups took the one-read backward
    assert fused_linear.STATS.get("residual LoRA", 0) == r0 + 1
    q0, u0 = mxfp8.STATS["quant"], mxfp8.STATS["reuse"]
    outs_m, dx_m, gr_m = _step(model, x, dys, dres, False)
    # module by module (_MXLinear): q/k/v share one input, quantized once and reused twice
    # (scripts/mxfp8.py:299-312); o_proj quantizes its own input; the backward quantizes each dy
    assert mxfp8.STATS["reuse"] - u0 >= 2
    assert mxfp8.STATS["quant"] - q0 >= 2
    errs = [_rel(a, b) for a, b in zip(outs_g, outs_m)] + [_rel(a, b) for a, b in zip(gr_g, gr_m)]
    assert max(errs) < TOL, errs
    # dx: the grouped path adds the three MX branches in fp32 inside one GEMM and rounds once; calling the
    # modules one by one rounds each branch (and each LoRA term) to bf16 and autograd adds them in bf16 --
    # the rounding-order difference the reference documents (scripts/fused_linear.py:9-11)
    assert _rel(dx_g, dx_m) < 1e-2
    mxfp8.disable_mxfp8(model)
    import _mxlib
    assert _mxlib.device_error() == 0
