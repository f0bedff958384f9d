"""Fused MXFP8 SwiGLU-LoRA MLP on the GPU vs the reference golden fixture and the CPU oracle.

Parity bar (BASELINE): forward outputs and LoRA gradients within a relative Frobenius error of 5e-3
of the dequantize-then-fp32-matmul oracle; MXFP8 codes / scales of h and [dg | du] byte-identical
except where exp() differs by an ulp between CUDA and numpy (a bounded, tiny fraction).
"""
import os

import numpy as np
import pytest
import torch

from oracle import mx_oracle as O

pytestmark = pytest.mark.gpu
TOL = 5e-3
G = os.path.join(os.path.dirname(__file__), "golden")
NAMES = ("dAg", "dBg", "dAu", "dBu", "dAd", "dBd")


def _bits_to_t(b):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


def _run(x, Wg, Wu, Wd, lora, dy, s, need_out=True):
    import fused_linear
    import fused_mlp
    fused_linear.new_step()     # the per-step bf16 cast cache is keyed by parameter id
    dev = torch.device("cuda")
    layer = fused_mlp.MXMLPWeights.from_bf16(Wg.to(dev), Wu.to(dev), Wd.to(dev))
    params = [p.to(dev).clone().requires_grad_(True) for p in lora]
    xd = x.to(dev).clone().requires_grad_(True)
    y = fused_mlp.mlp_apply(layer, xd, *params, scaling=(s, s, s), need_out=need_out)
    y.backward(dy.to(dev))
    torch.cuda.synchronize()
    import _mxlib
    assert _mxlib.device_error() == 0
    return y.detach().float().cpu(), xd.grad.float().cpu(), [p.grad.float().cpu() for p in params]


def _case(T, H, N, r, seed, outlier=0.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g)
    if outlier:
        x = torch.where(torch.rand(T, H, generator=g) < 0.01, x * outlier, x)
    x = x.to(torch.bfloat16)
    Wg = (torch.randn(N, H, generator=g) * 0.02).to(torch.bfloat16)
    Wu = (torch.randn(N, H, generator=g) * 0.02).to(torch.bfloat16)
    Wd = (torch.randn(H, N, generator=g) * 0.02).to(torch.bfloat16)
    lora = [torch.randn(*sh, generator=g) * 0.01 for sh in ((r, H), (N, r), (r, H), (N, r), (r, N), (H, r))]
    dy = torch.randn(T, H, generator=g).to(torch.bfloat16)
    return x, Wg, Wu, Wd, lora, dy


def _oracle(x, Wg, Wu, Wd, lora, dy, s):
    W = O.MXWeights(Wg.float().numpy(), Wu.float().numpy(), Wd.float().numpy())
    yo, ctx = O.mlp_forward(x.float().numpy(), W, *[p.numpy() for p in lora], s, s, s)
    go = O.mlp_backward(dy.float().numpy(), ctx)
    return yo, go, ctx


def test_mlp_vs_reference_golden():
    z = np.load(os.path.join(G, "mlp_golden.npz"))
    x, dy = _bits_to_t(z["x"]), _bits_to_t(z["dy"])
    Wg, Wu, Wd = (_bits_to_t(z[k]) for k in ("Wg", "Wu", "Wd"))
    lora = [torch.from_numpy(z[k]) for k in ("Ag", "Bg", "Au", "Bu", "Ad", "Bd")]
    s = float(z["alpha"]) / float(z["r"])
    y, dx, grads = _run(x, Wg, Wu, Wd, lora, dy, s)
    assert O.rel_fro(y.numpy(), O.bf16_bits_to_f32(z["y"])) < TOL
    assert O.rel_fro(dx.numpy(), O.bf16_bits_to_f32(z["dx"])) < TOL
    for gr, k in zip(grads, NAMES):
        assert O.rel_fro(gr.numpy(), z[k]) < TOL, k


@pytest.mark.parametrize("T", [512, 1, 77, 1000, 2049])
def test_mlp_08b_shape_vs_oracle(T):
    """0.8B MLP shape (hidden 1024, intermediate 3584, r 16, alpha 32), ragged token counts."""
    H, N, r, s = 1024, 3584, 16, 2.0
    case = _case(T, H, N, r, seed=T, outlier=100.0 if T != 512 else 0.0)
    y, dx, grads = _run(*case, s)
    yo, go, _ = _oracle(*case, s)
    assert O.rel_fro(y.numpy(), yo) < TOL
    assert O.rel_fro(dx.numpy(), go["dx"]) < TOL
    for gr, k in zip(grads, NAMES):
        assert O.rel_fro(gr.numpy(), go[k]) < TOL, (k, O.rel_fro(gr.numpy(), go[k]))


def test_mlp_rank32():
    T, H, N, r, s = 300, 512, 1024, 32, 1.0
    case = _case(T, H, N, r, seed=5)
    y, dx, grads = _run(*case, s)
    yo, go, _ = _oracle(*case, s)
    assert O.rel_fro(y.numpy(), yo) < TOL
    assert O.rel_fro(dx.numpy(), go["dx"]) < TOL
    for gr, k in zip(grads, NAMES):
        assert O.rel_fro(gr.numpy(), go[k]) < TOL, k


def test_epilogue_bytes_vs_oracle():
    """h's and [dg | du]'s MXFP8 bytes from the CUDA epilogues vs the oracle on the same gu / dh."""
    import fused_linear
    import fused_mlp
    fused_linear.new_step()
    T, H, N, r, s = 333, 512, 1024, 16, 2.0
    x, Wg, Wu, Wd, lora, dy = _case(T, H, N, r, seed=11)
    yo, go, ctx = _oracle(x, Wg, Wu, Wd, lora, dy, s)
    dev = torch.device("cuda")
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(dev)  # noqa: E731
    gu, xs = bf(ctx["gu"]), bf(ctx["xs"])
    bg, bu, ad = bf(ctx["bg"]), bf(ctx["bu"]), bf(ctx["ad"])
    qh, sh, xsd = fused_mlp.mlp_fwd(gu, xs, bg, bu, ad, s, s, True)
    torch.cuda.synchronize()
    dq = (qh.view(torch.uint8).cpu().numpy() != ctx["qh"]).mean()
    ds = (sh.view(torch.uint8).cpu().numpy() != ctx["sh"]).mean()
    assert dq < 1e-3 and ds < 1e-3, (dq, ds)
    assert O.rel_fro(xsd.float().cpu().numpy(), ctx["xsd"]) < 2e-3
    q, sc, dxa, dbg, dbu, dad = fused_mlp.mlp_bwd(gu, xs, bf(go["dhm"]), bf(go["dxd"]), bg, bu, ad, s, s, True)
    torch.cuda.synchronize()
    dq = (q.view(torch.uint8).cpu().numpy() != go["q_dgu"]).mean()
    ds = (sc.view(torch.uint8).cpu().numpy() != go["s_dgu"]).mean()
    assert dq < 1e-3 and ds < 1e-3, (dq, ds)
    assert O.rel_fro(dbg.cpu().numpy() * s, go["dBg"]) < 2e-3
    assert O.rel_fro(dbu.cpu().numpy() * s, go["dBu"]) < 2e-3
    assert O.rel_fro(dad.cpu().numpy(), go["dAd"]) < 2e-3


def test_need_out_false_and_determinism():
    """need_out=False (checkpoint recompute) gives the same gradients; two runs are bitwise equal."""
    T, H, N, r, s = 640, 1024, 3584, 16, 2.0
    case = _case(T, H, N, r, seed=9)
    y1, dx1, g1 = _run(*case, s)
    y2, dx2, g2 = _run(*case, s)
    assert torch.equal(y1, y2) and torch.equal(dx1, dx2)
    assert all(torch.equal(a, b) for a, b in zip(g1, g2))
    _, dx3, g3 = _run(*case, s, need_out=False)
    assert torch.equal(dx1, dx3)
    assert all(torch.equal(a, b) for a, b in zip(g1, g3))


@pytest.mark.parametrize("T,H,N", [(1, 1024, 3584), (77, 1024, 3584), (1000, 2048, 6144), (2049, 1024, 3584),
                                   (4096, 2048, 6144)])
def test_gemm_glu_matches_two_passes(T, H, N):
    """The gate|up GEMM with the fused forward epilogue gives the same MXFP8(h) bytes as the GEMM followed by
    the separate epilogue kernel, and gu = [g | u] = bf16(GEMM + s xa B^T) (the two-pass gu plus the LoRA
    terms, up to the fp32 summation order of the rank-16 dot); xS_down differs only by that order too.
    T >= 256 runs the CTA-pair kernel (2049: an odd count of 128-row blocks, so the last pair's second CTA
    holds no rows), smaller T the single-CTA kernel."""
    import fused_mlp
    import mxfp8
    g = torch.Generator().manual_seed(T + N)
    dev = torch.device("cuda")
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(2 * N, H, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    r = 16
    xs = (torch.randn(T, 2 * r, generator=g) * 0.5).to(torch.bfloat16).to(dev)
    bg = (torch.randn(N, r, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    bu = (torch.randn(N, r, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    ad = (torch.randn(r, N, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    q, sc = mxfp8.mx_quant(x)
    qw, sw = mxfp8.mx_quant(w)
    gu, qh, sh, xsd = fused_mlp.gemm_glu(q, sc, qw, sw, xs, bg, bu, ad, 2.0, 2.0)
    gu0 = mxfp8.mx_mm(q, qw.t(), sc, sw)
    qh0, sh0, xsd0 = fused_mlp.mlp_fwd(gu0, xs, bg, bu, ad, 2.0, 2.0, True)
    torch.cuda.synchronize()
    import _mxlib
    assert _mxlib.device_error() == 0
    lora = torch.cat([xs[:, :r].float() @ bg.float().t(), xs[:, r:].float() @ bu.float().t()], 1)
    mag = torch.cat([xs[:, :r].float().abs() @ bg.float().abs().t(), xs[:, r:].float().abs() @ bu.float().abs().t()], 1)
    ref = (gu0.float() + 2.0 * lora).to(torch.bfloat16)
    assert float((gu != ref).float().mean()) < 1e-3
    # one bf16 rounding apart, where the rank-16 dot may cancel: bounded by the magnitudes it sums
    bound = (ref.float().abs() + gu0.float().abs() + 2.0 * mag) * 2.0 ** -7
    assert bool(((gu.float() - ref.float()).abs() <= bound).all())
    assert torch.equal(qh.view(torch.uint8), qh0.view(torch.uint8))
    assert torch.equal(sh.view(torch.uint8), sh0.view(torch.uint8))
    d = (xsd.float() - xsd0.float()).abs()
    assert float(d.max()) <= float(xsd0.float().abs().max()) * 2.0 ** -7 + 1e-6
    assert float((xsd != xsd0).float().mean()) < 0.01


@pytest.mark.parametrize("T", [77, 2049])
def test_cuda_graph_replay_matches_eager(T):
    """One fused fwd+bwd captured in a CUDA graph (static inputs) and replayed gives exactly the eager
    step's output and gradients: the path makes no host synchronisation and no allocation outside
    torch's allocator, so small-M callers can graph it (bench.py --workload ragged)."""
    import fused_linear
    import fused_mlp
    H, N, r, s = 1024, 3584, 16, 2.0
    x, Wg, Wu, Wd, lora, dy = _case(T, H, N, r, seed=T + 5, outlier=100.0)
    dev = torch.device("cuda")
    layer = fused_mlp.MXMLPWeights.from_bf16(Wg.to(dev), Wu.to(dev), Wd.to(dev))
    params = [p.to(dev).clone().requires_grad_(True) for p in lora]
    xs, dys = x.to(dev), dy.to(dev)
    out = {}

    def step():
        fused_linear.new_step()
        h = xs.detach().requires_grad_(True)
        y = fused_mlp.mlp_apply(layer, h, *params, scaling=(s, s, s))
        y.backward(dys)
        out["y"], out["dx"] = y.detach(), h.grad   # no reference to the autograd graph survives the step

    step()
    torch.cuda.synchronize()
    ref = [out["y"].clone(), out["dx"].clone()] + [p.grad.clone() for p in params]
    for p in params:
        p.grad = None
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
            for p in params:
                p.grad = None
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    got = [out["y"], out["dx"]] + [p.grad for p in params]
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    import _mxlib
    assert _mxlib.device_error() == 0


def _codes_differ(a, b):
    """Share of E4M3 codes that differ (two NaN codes count as equal)."""
    a, b = np.asarray(a, np.uint8), np.asarray(b, np.uint8)
    nan = ((a & 0x7F) == 0x7F) & ((b & 0x7F) == 0x7F)
    return float(((a != b) & ~nan).mean())


@pytest.mark.parametrize("T", [1024, 2049, 4352])
def test_mlp_2b_shape_vs_oracle(T):
    """The benchmarked shape (Qwen3.5-2B MLP: hidden 2048, intermediate 6144, r 16, alpha 32): y, dx and
    all six LoRA gradients within 5e-3 of the oracle.  T = 2049 is an odd count of 128-row blocks, so the
    CTA-pair gate|up kernel's last pair has a second CTA without rows."""
    H, N, r, s = 2048, 6144, 16, 2.0
    case = _case(T, H, N, r, seed=20000 + T, outlier=100.0)
    y, dx, grads = _run(*case, s)
    yo, go, _ = _oracle(*case, s)
    assert O.rel_fro(y.numpy(), yo) < TOL
    assert O.rel_fro(dx.numpy(), go["dx"]) < TOL
    for gr, k in zip(grads, NAMES):
        assert O.rel_fro(gr.numpy(), go[k]) < TOL, (k, O.rel_fro(gr.numpy(), go[k]))


@pytest.mark.parametrize("T", [1024, 2049])
def test_epilogue_bytes_2b_vs_oracle(T):
    """At the 2B shape, the kernels the step runs -- the gate|up GEMM with the fused forward epilogue and
    the backward epilogue -- against the oracle's epilogues fed the same gu / dh_mx: MXFP8(h) and
    MXFP8([dg | du]) codes and scales equal except where exp / reciprocal differ by an ulp (< 1e-3 of the
    codes), the partial products within 2e-3."""
    import fused_linear
    import fused_mlp
    import mxfp8
    fused_linear.new_step()
    H, N, r, s = 2048, 6144, 16, 2.0
    x, Wg, Wu, Wd, lora, dy = _case(T, H, N, r, seed=30000 + T, outlier=100.0)
    dev = torch.device("cuda")
    layer = fused_mlp.MXMLPWeights.from_bf16(Wg.to(dev), Wu.to(dev), Wd.to(dev))
    P = fused_mlp.lora_prep(*(p.to(dev) for p in (lora[0], lora[2], lora[1], lora[3], lora[4], lora[5])), s)
    S, bg, bu, ad, bd, bds, bdT, ST = P
    xd, dyd = x.to(dev), dy.to(dev)
    xs, q, sc = fused_mlp.rowdot_quant(xd, S)
    gu, qh, sh, xsd = fused_mlp.gemm_glu(q, sc, layer.hold.w, layer.hold.ws, xs, bg, bu, ad, s, s)
    gu0 = mxfp8.mx_mm(q, layer.hold.w.t(), sc, layer.hold.ws)   # the GEMM alone: the oracle's input
    dxd, qd, sd = fused_mlp.rowdot_quant(dyd, bdT, post=s)
    wt, wts = mxfp8.mx_wt(layer.down)
    dhm = mxfp8.mx_mm(qd, wt.t(), sd, wts)
    qg, sg, dxa, dbg, dbu, dad = fused_mlp.mlp_bwd(gu, xs, dhm, dxd, bg, bu, ad, s, s, True, gu_lora=True)
    torch.cuda.synchronize()
    import _mxlib
    assert _mxlib.device_error() == 0
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    g_o, u_o = O._gu(f(gu0), f(xs), f(bg), f(bu), s, s, N, r)   # the fused kernel's gu holds g | u
    assert float((f(gu) != np.concatenate([g_o, u_o], 1)).mean()) < 1e-3
    h_o, qh_o, sh_o, xsd_o = O.fwd_epilogue(f(gu0), f(xs), f(bg), f(bu), f(ad), s, s)
    assert _codes_differ(qh.view(torch.uint8).cpu().numpy(), qh_o) < 1e-3
    assert float((sh.view(torch.uint8).cpu().numpy() != sh_o).mean()) < 1e-3
    assert O.rel_fro(f(xsd), xsd_o) < 2e-3
    e = O.bwd_epilogue(f(gu0), f(xs), f(dhm), f(dxd), f(bg), f(bu), f(ad), s, s)
    assert _codes_differ(qg.view(torch.uint8).cpu().numpy(), e["q_dgu"]) < 1e-3
    assert float((sg.view(torch.uint8).cpu().numpy() != e["s_dgu"]).mean()) < 1e-3
    assert O.rel_fro(f(dbg), e["dBg"]) < 2e-3 and O.rel_fro(f(dbu), e["dBu"]) < 2e-3
    assert O.rel_fro(f(dad), e["dAd"]) < 2e-3
    assert O.rel_fro(f(dxa)[:, :r], e["dxa_g"]) < 2e-3 and O.rel_fro(f(dxa)[:, r:2 * r], e["dxa_u"]) < 2e-3
    assert O.rel_fro(f(dxa)[:, 2 * r:], e["xsd"]) < 2e-3


@pytest.mark.parametrize("T,gu_lora", [(300, False), (4352, False), (4352, True)])
def test_bwd_epilogue_without_codes(T, gu_lora):
    """need_q = False (x needs no gradient): the backward epilogue skips the MXFP8 of [dg | du] and gives the
    same partial products, bit for bit, as the run that writes the codes (those are checked against the
    oracle above).  T = 300 leaves the last 256-row block mostly empty; 4352 = 17 blocks of 256."""
    import fused_mlp
    H, N, r, s = 2048, 6144, 16, 2.0
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(T)
    gu = (torch.randn(T, 2 * N, generator=g) * 2).to(torch.bfloat16).to(dev)
    xs = torch.randn(T, 2 * r, generator=g).to(torch.bfloat16).to(dev)
    dhm = (torch.randn(T, N, generator=g) * 0.01).to(torch.bfloat16).to(dev)
    dxd = (torch.randn(T, r, generator=g) * 0.01).to(torch.bfloat16).to(dev)
    bg, bu = ((torch.randn(N, r, generator=g) * 0.05).to(torch.bfloat16).to(dev) for _ in range(2))
    ad = (torch.randn(r, N, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    with_q = fused_mlp.mlp_bwd(gu, xs, dhm, dxd, bg, bu, ad, s, s, True, gu_lora=gu_lora)
    no_q = fused_mlp.mlp_bwd(gu, xs, dhm, dxd, bg, bu, ad, s, s, False, gu_lora=gu_lora)
    torch.cuda.synchronize()
    import _mxlib
    assert _mxlib.device_error() == 0
    assert no_q[0] is None and no_q[1] is None
    for a, b in zip(with_q[2:], no_q[2:]):
        assert torch.equal(a, b)


def test_configs0_exact():
    """configs[0] as BASELINE states it: 0.8B MLP shape, X bf16 [512, 1024] ~ N(0,1); W_gate, W_up
    [3584, 1024] and W_down [1024, 3584] ~ N(0, 0.02); LoRA r 16, alpha 32 on all three with A, B ~
    N(0, 0.01); dY ~ N(0,1) bf16; seed 0 (one torch generator, drawn in that order)."""
    T, H, N, r, s = 512, 1024, 3584, 16, 2.0
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    Wg = (torch.randn(N, H, generator=g) * 0.02).to(torch.bfloat16)
    Wu = (torch.randn(N, H, generator=g) * 0.02).to(torch.bfloat16)
    Wd = (torch.randn(H, N, generator=g) * 0.02).to(torch.bfloat16)
    lora = [torch.randn(*sh, generator=g) * 0.01 for sh in ((r, H), (N, r), (r, H), (N, r), (r, N), (H, r))]
    dy = torch.randn(T, H, generator=g).to(torch.bfloat16)
    case = (x, Wg, Wu, Wd, lora, dy)
    y, dx, grads = _run(*case, s)
    yo, go, _ = _oracle(*case, s)
    assert O.rel_fro(y.numpy(), yo) < TOL
    assert O.rel_fro(dx.numpy(), go["dx"]) < TOL
    for gr, k in zip(grads, NAMES):
        assert O.rel_fro(gr.numpy(), go[k]) < TOL, (k, O.rel_fro(gr.numpy(), go[k]))


def test_ragged_10752_vs_oracle():
    """configs[4]'s largest ragged M (10752 = 84 blocks of 128, not a multiple of 256) at the 0.8B shape
    with 1 % x100 outliers."""
    T, H, N, r, s = 10752, 1024, 3584, 16, 2.0
    case = _case(T, H, N, r, seed=10752, outlier=100.0)
    y, dx, grads = _run(*case, s)
    yo, go, _ = _oracle(*case, s)
    assert O.rel_fro(y.numpy(), yo) < TOL
    assert O.rel_fro(dx.numpy(), go["dx"]) < TOL
    for gr, k in zip(grads, NAMES):
        assert O.rel_fro(gr.numpy(), go[k]) < TOL, (k, O.rel_fro(gr.numpy(), go[k]))
