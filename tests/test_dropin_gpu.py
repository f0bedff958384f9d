"""The drop-in entry as the reference's caller uses it: ``mxfp8.enable_mxfp8(model)`` on a model whose MLP
projections are PEFT LoRA layers, then ``fused_mlp.mlp(layer.mlp, x, need_out)`` (the caller's code at
scripts/shared_prefix.py:189-193; gate/up pairing at scripts/mxfp8.py:472-484; gating at
scripts/fused_mlp.py:343-366).  The output and every gradient are checked against the oracle, and each
case where the reference returns None (so the caller runs its unfused path) returns None here too.

PEFT is not installed in this image, so ``LoraLinear`` below carries exactly the attributes of a PEFT
``lora.Linear`` that the entry reads (base_layer, lora_A / lora_B / lora_dropout ModuleDicts, scaling,
use_dora, merged, disable_adapters, active_adapters).
"""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import mx_oracle as O

pytestmark = pytest.mark.gpu
TOL = 5e-3


class LoraLinear(nn.Module):
    def __init__(self, base, r, alpha):
        super().__init__()
        self.base_layer = base
        self.lora_A = nn.ModuleDict({"default": nn.Linear(base.in_features, r, bias=False)})
        self.lora_B = nn.ModuleDict({"default": nn.Linear(r, base.out_features, bias=False)})
        self.lora_dropout = nn.ModuleDict({"default": nn.Identity()})
        self.scaling = {"default": alpha / r}
        self.use_dora = {"default": False}
        self.merged = False
        self.disable_adapters = False
        self.active_adapters = ["default"]

    def forward(self, x):
        a = "default"
        return self.base_layer(x) + self.lora_B[a](self.lora_A[a](self.lora_dropout[a](x))) * self.scaling[a]


class MLP(nn.Module):
    def __init__(self, H, N, r, alpha, g):
        super().__init__()
        def lin(i, o):
            m = nn.Linear(i, o, bias=False)
            m.weight.data = (torch.randn(o, i, generator=g) * 0.02).to(torch.bfloat16)
            m.weight.requires_grad_(False)
            return m
        self.gate_proj = LoraLinear(lin(H, N), r, alpha)
        self.up_proj = LoraLinear(lin(H, N), r, alpha)
        self.down_proj = LoraLinear(lin(N, H), r, alpha)
        for m in (self.gate_proj, self.up_proj, self.down_proj):
            for d in (m.lora_A, m.lora_B):
                w = d["default"].weight
                w.data = torch.randn(w.shape, generator=g) * 0.01


class Block(nn.Module):
    def __init__(self, *a):
        super().__init__()
        self.mlp = MLP(*a)


class Model(nn.Module):
    def __init__(self, H, N, r, alpha, seed, n_layers=1):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.model = nn.Module()
        self.model.layers = nn.ModuleList([Block(H, N, r, alpha, g) for _ in range(n_layers)])


def _model(H=1024, N=3584, r=16, alpha=32, seed=3, n_layers=1):
    return Model(H, N, r, alpha, seed, n_layers).cuda()


def _oracle_of(mlp, x, dy, s):
    """Oracle forward + backward on the module's (bf16 base, fp32 LoRA) weights, before enable_mxfp8 moves
    the bf16 weights to the host."""
    W = O.MXWeights(*(m.base_layer.weight.float().cpu().numpy() for m in (mlp.gate_proj, mlp.up_proj, mlp.down_proj)))
    lora = []
    for m in (mlp.gate_proj, mlp.up_proj, mlp.down_proj):
        lora += [m.lora_A["default"].weight.detach().cpu().numpy(), m.lora_B["default"].weight.detach().cpu().numpy()]
    yo, ctx = O.mlp_forward(x.reshape(-1, x.shape[-1]).float().cpu().numpy(), W, *lora, s, s, s)
    go = O.mlp_backward(dy.reshape(-1, dy.shape[-1]).float().cpu().numpy(), ctx)
    return yo, go


def _lora_params(mlp):
    return [m.lora_A["default"].weight if k == 0 else m.lora_B["default"].weight
            for m in (mlp.gate_proj, mlp.up_proj, mlp.down_proj) for k in (0, 1)]


def test_mlp_entry_after_enable_mxfp8_matches_oracle():
    import fused_linear
    import fused_mlp
    import mxfp8
    model = _model()
    mlp = model.model.layers[0].mlp
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 300, 1024, generator=g).to(torch.bfloat16).cuda()   # [B, T, H]: leading dims kept
    dy = torch.randn(2, 300, 1024, generator=g).to(torch.bfloat16).cuda()
    yo, go = _oracle_of(mlp, x, dy, 2.0)
    n = mxfp8.enable_mxfp8(model)
    try:
        assert n == 3
        gb, ub = mlp.gate_proj.base_layer, mlp.up_proj.base_layer
        hold = gb._mx_gu[0]
        assert ub._mx_gu == (hold, 1) and gb._mx_gu == (hold, 0) and mxfp8.is_mx(mlp.down_proj.base_layer)
        assert gb.weight.numel() == 0 and gb._bf16_cpu.shape == (3584, 1024)
        before = fused_mlp.STATS.get("mlp gộp", 0)
        fused_mlp.ACTIVE[0] = False
        fused_linear.new_step()
        xg = x.clone().requires_grad_(True)
        y = fused_mlp.mlp(mlp, xg, True)
        assert y is not None and y.shape == x.shape and y.dtype == torch.bfloat16
        assert fused_mlp.STATS["mlp gộp"] == before + 1 and fused_mlp.ACTIVE[0]
        y.backward(dy)
        torch.cuda.synchronize()
        assert O.rel_fro(y.detach().float().cpu().numpy().reshape(-1, 1024), yo) < TOL
        assert O.rel_fro(xg.grad.float().cpu().numpy().reshape(-1, 1024), go["dx"]) < TOL
        for p, k in zip(_lora_params(mlp), ("dAg", "dBg", "dAu", "dBu", "dAd", "dBd")):
            assert p.grad is not None and p.grad.dtype == torch.float32
            assert O.rel_fro(p.grad.cpu().numpy(), go[k]) < TOL, k
    finally:
        mxfp8.disable_mxfp8(model)
    # disable_mxfp8 restores the bf16 weights on the device and removes every attribute it added
    assert mlp.gate_proj.base_layer.weight.shape == (3584, 1024) and mlp.gate_proj.base_layer.weight.is_cuda
    for a in ("_mx_w", "_mx_ws", "_mx_gu", "_bf16_cpu", "forward"):
        assert a not in mlp.gate_proj.base_layer.__dict__


def test_mlp_entry_autocast_and_need_out_false():
    """Under bf16 autocast an fp32 input takes the fused path (the compute dtype is autocast's); with
    need_out=False the gradients are the same as with need_out=True (checkpoint recompute)."""
    import fused_linear
    import fused_mlp
    import mxfp8
    model = _model(seed=4)
    mlp = model.model.layers[0].mlp
    g = torch.Generator().manual_seed(6)
    x = torch.randn(200, 1024, generator=g).to(torch.bfloat16).float().cuda()
    dy = torch.randn(200, 1024, generator=g).to(torch.bfloat16).cuda()
    mxfp8.enable_mxfp8(model)
    try:
        res = []
        for need_out in (True, False):
            fused_linear.new_step()
            for p in _lora_params(mlp):
                p.grad = None
            xg = x.clone().requires_grad_(True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                y = fused_mlp.mlp(mlp, xg, need_out)
            assert y is not None
            y.backward(dy)
            torch.cuda.synchronize()
            assert xg.grad.dtype == torch.float32       # dx back in x's dtype
            res.append([xg.grad.clone()] + [p.grad.clone() for p in _lora_params(mlp)])
        for a, b in zip(*res):
            assert torch.equal(a, b)
    finally:
        mxfp8.disable_mxfp8(model)


def test_mlp_entry_returns_none_where_the_reference_does():
    import fused_mlp
    import mxfp8
    x = torch.randn(64, 1024).to(torch.bfloat16).cuda()
    # rank 64: not a rank the fused kernels take
    model = _model(r=64, alpha=64, seed=7)
    mxfp8.enable_mxfp8(model)
    try:
        assert fused_mlp.mlp(model.model.layers[0].mlp, x) is None
    finally:
        mxfp8.disable_mxfp8(model)
    model = _model(seed=8)
    mlp = model.model.layers[0].mlp
    mxfp8.enable_mxfp8(model)
    try:
        assert fused_mlp.mlp(mlp, x.float()) is None                 # fp32 compute dtype (no autocast)
        assert fused_mlp.mlp(mlp, x.cpu()) is None                   # not on CUDA
        fused_mlp.ENABLED[0] = False
        try:
            assert fused_mlp.mlp(mlp, x) is None                     # switched off
        finally:
            fused_mlp.ENABLED[0] = True
        mlp.up_proj.lora_dropout["default"] = nn.Dropout(0.1)         # a dropout the fused path does not do
        assert fused_mlp.mlp(mlp, x) is None
        mlp.up_proj.lora_dropout["default"] = nn.Identity()
        assert fused_mlp.mlp(mlp, x) is not None
    finally:
        mxfp8.disable_mxfp8(model)
    # gate and up quantized separately (the reference's MXFP8_FUSE_GU=0): no shared gate|up pair
    model = _model(seed=9)
    saved = mxfp8.FUSE_GU
    mxfp8.FUSE_GU = False
    try:
        mxfp8.enable_mxfp8(model)
        mlp = model.model.layers[0].mlp
        assert "_mx_gu" not in mlp.gate_proj.base_layer.__dict__ and mxfp8.is_mx(mlp.gate_proj.base_layer)
        assert fused_mlp.mlp(mlp, x) is None
    finally:
        mxfp8.FUSE_GU = saved
        mxfp8.disable_mxfp8(model)
