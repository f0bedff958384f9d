"""The whole MLP (gate/up + SwiGLU + LoRA + MX quantization + dB/dxa/dA) in ONE autograd.Function, on
B200 (sm_100a) kernels.  Drop-in for the reference module of the same name (scripts/fused_mlp.py):
same globals (``ENABLED``, ``ACTIVE``, ``SAVED_LESS``, ``STATS``), entry point ``mlp(mlp_mod, x,
need_out)``, ``_MLP`` autograd contract (9 inputs, 9 gradients, the same saved tensors in both
``need_out`` modes) and ``mlp_fwd`` / ``mlp_bwd`` helpers.

Per layer call (T tokens, H hidden, N intermediate, r LoRA rank):
  forward : xs = x S^T (rank-2r, tensor-core rowdot) and q, s = MXFP8(x) from one read of x
            gu = [x W_gate^T | x W_up^T]          -- tcgen05 block-scaled GEMM, K = H, and in the same
            q_h, s_h, xS_down = epilogue(gu)          kernel (rank 16) the LoRA-B add, SwiGLU, MX quantize h
            y = h W_down^T + xS_down (s_d B_down)^T -- tcgen05 GEMM; the LoRA term is a bf16 tcgen05 MMA
                                                       into the same TMEM accumulator
  backward: q, s = MXFP8(dy) and dxd = s_d dy B_down from one read of dy; dh_mx = dy W_down (tcgen05)
            [dg | du] MXFP8 + dB_g, dB_u, dA_d, dxa, xS_down = epilogue(gu, dh_mx)
            dx = [dg | du] W_gu + dxa S (tcgen05 GEMM, K = 2N, LoRA term as a bf16 MMA)
            dB_d = s_d dy^T xS_down;  dA = dxa^T x (tensor-core coldot)
The math and the bf16 rounding points follow the reference (scripts/fused_mlp.py:262-336), except that y
and dx are rounded to bf16 once after the LoRA add (the reference rounds the MX product first), and the
fp32 summation order.  h is not saved (the backward recomputes it from gu).
"""
import types

import torch

import _mxlib as _nx
import mx_dp
import mxfp8
from fused_linear import STATS, _cast, _part

_F8, _E8 = torch.float8_e4m3fn, torch.float8_e8m0fnu
ENABLED = [True]    # set False to compare against the unfused path in the same process
ACTIVE = [False]    # the fused path ran at least once (read by the caller's activation budgeting)
SAVED_LESS = 12288  # bytes per token per layer no longer saved versus the unfused path (h [T, 6144] bf16)


def _cdiv(a, b):
    return -(-a // b)


# ------------------------------------------------------------------------------------------------ skinny ops
def rowdot(A, B, post=1.0, out=None):
    """bf16(bf16(A @ B^T) * post): A [T, K] bf16 (K % 32 == 0), B [n, K] bf16 contiguous, n in {16, 32}."""
    T, K = A.shape
    n = B.shape[0]
    assert A.stride(1) == 1 and B.is_contiguous() and B.shape[1] == K
    if out is None:
        out = torch.empty((T, n), dtype=torch.bfloat16, device=A.device)
    _nx.call("mxm_rowdot", _nx.ptr(A), A.stride(0), _nx.ptr(B), T, K, n, float(post), _nx.ptr(out), out.stride(0),
             _nx.stream_of(A))
    return out


def rowdot_quant(A, B, post=1.0):
    """(rowdot(A, B, post), *mxfp8.mx_quant(A)) from one read of A: A [T, K] bf16 contiguous, K % 128 == 0."""
    T, K = A.shape
    n = B.shape[0]
    assert A.is_contiguous() and B.is_contiguous() and B.shape[1] == K
    out = torch.empty((T, n), dtype=torch.bfloat16, device=A.device)
    q = torch.empty((T, K), dtype=_F8, device=A.device)
    s = torch.empty(mxfp8.scale_numel(T, K), dtype=torch.uint8, device=A.device)
    _nx.call("mxm_rowdot_quant", _nx.ptr(A), K, _nx.ptr(B), T, K, n, float(post), _nx.ptr(out), out.stride(0),
             _nx.ptr(q), K, _nx.ptr(s), _nx.stream_of(A))
    return out, q, s.view(_E8)


def coldot(A, E, post=1.0, transpose_out=False, out_dtype=torch.bfloat16, out=None):
    """bf16(bf16(A^T @ E) * post): A [T, K] bf16, E [T, n] bf16 (n in {16, 32, 64}) -> [K, n] (or [n, K]);
    out_dtype float32 stores the same bf16-valued numbers in fp32 (a gradient for an fp32 parameter).
    `out`: a contiguous destination of that shape and dtype (else one is allocated)."""
    T, K = A.shape
    n = E.shape[1]
    assert out_dtype in (torch.bfloat16, torch.float32)
    rpc, nch = _nx.coldot_chunks(T, K)
    part = torch.empty((nch, K, n), dtype=torch.float32, device=A.device)
    shape = (n, K) if transpose_out else (K, n)
    if out is None:
        out = torch.empty(shape, dtype=out_dtype, device=A.device)
    assert out.shape == shape and out.dtype == out_dtype and out.is_contiguous(), (out.shape, out.dtype)
    _nx.call("mxm_coldot", _nx.ptr(A), A.stride(0), _nx.ptr(E), E.stride(0), T, K, n, float(post),
             1 if transpose_out else 0, _nx.ptr(part), rpc, nch, _nx.ptr(out),
             1 if out_dtype == torch.float32 else 0, _nx.stream_of(A))
    return out


def lora_prep(Ag, Au, Bg, Bu, Ad, Bd, s_d):
    """The bf16 LoRA operands of one step in one launch: (S, bg, bu, ad, bd, bds, bdT, ST) with
    S = [Ag; Au], bds = bf16(bd * s_d), bdT = bd^T, ST = S^T (all contiguous views of one buffer); None
    when the parameters are not all contiguous fp32 or all contiguous bf16 on one device."""
    ws = (Ag, Au, Bg, Bu, Ad, Bd)
    dts = {w.dtype for w in ws}
    if len(dts) != 1 or dts.pop() not in (torch.float32, torch.bfloat16) or \
            not all(w.is_contiguous() and w.device == Ag.device for w in ws):
        return None
    r, H = Ag.shape
    N = Bg.shape[0]
    if Au.shape != (r, H) or Bg.shape != (N, r) or Bu.shape != (N, r) or Ad.shape != (r, N) or Bd.shape != (H, r):
        return None
    buf = torch.empty(r * (7 * H + 3 * N), dtype=torch.bfloat16, device=Ag.device)
    _nx.call("mxm_lora_prep", _nx.ptr(Ag), _nx.ptr(Au), _nx.ptr(Bg), _nx.ptr(Bu), _nx.ptr(Ad), _nx.ptr(Bd),
             1 if Ag.dtype == torch.float32 else 0, H, N, r, float(s_d), _nx.ptr(buf), _nx.stream_of(Ag))
    sizes = [2 * r * H, N * r, N * r, r * N, H * r, H * r, r * H, H * 2 * r]
    shapes = [(2 * r, H), (N, r), (N, r), (r, N), (H, r), (H, r), (r, H), (H, 2 * r)]
    return tuple(p.view(sh) for p, sh in zip(torch.split(buf, sizes), shapes))


# the MX GEMM with the LoRA term in its accumulator (mxfp8.mx_mm_lora); a module-level name so that callers
# and benchmarks can reach it as fused_mlp.mx_mm_lora
mx_mm_lora = mxfp8.mx_mm_lora


# ------------------------------------------------------------------------------------------------ epilogues
def mlp_fwd(gu, xs, bg, bu, ad, s_g, s_u, write_q):
    """gu [T, 2N] bf16, xs [T, 2R] bf16 (xa_gate | xa_up), bg / bu [N, R], ad [R, N] bf16 ->
    (q_h, s_h, xS_down bf16) -- scripts/fused_mlp.py:198-215."""
    T, N2 = gu.shape
    N, R = N2 // 2, ad.shape[0]
    dev = gu.device
    cs = _nx.mlp_fwd_partitions(T, N, R)
    q = s = None
    if write_q:
        q = torch.empty((T, N), dtype=_F8, device=dev)
        s = torch.empty(_cdiv(T, 128) * (N // 128) * 512, dtype=torch.uint8, device=dev)
    xsd = torch.empty((T, R), dtype=torch.bfloat16, device=dev)
    part = torch.empty((cs, T, R), dtype=torch.float32, device=dev) if cs > 1 else None
    _nx.call("mxm_mlp_fwd_epilogue", _nx.ptr(gu), _nx.ptr(xs), _nx.ptr(bg), _nx.ptr(bu), _nx.ptr(ad), T, N, R,
             float(s_g), float(s_u), _nx.ptr(q), _nx.ptr(s), _nx.ptr(xsd), _nx.ptr(part), cs, _nx.stream_of(gu))
    return (q, s.view(_E8), xsd) if write_q else (None, None, xsd)


def gemm_glu(q, sc, w, ws, xs, bg, bu, ad, s_g, s_u):
    """The gate|up GEMM and, from the same tiles, the forward epilogue (MXFP8(h), xS_down): mx_mm + mlp_fwd
    in one kernel.  q / sc: MXFP8(x) [T, H]; w / ws: W_gu codes [2N, H] and scales.
    -> (gu [T, 2N] bf16 = [g | u] with the LoRA terms added -- the values the SwiGLU used, which the
    backward takes with gu_lora=True --, q_h [T, N] fp8, s_h, xS_down [T, r] bf16).  Rank 16 only."""
    T, H = q.shape
    N2 = w.shape[0]
    N, R = N2 // 2, ad.shape[0]
    dev = q.device
    per, grid, slots = _nx.glu_partition(T, N)
    gu = torch.empty((T, N2), dtype=torch.bfloat16, device=dev)
    qh = torch.empty((T, N), dtype=_F8, device=dev)
    sh = torch.empty(_cdiv(T, 128) * (N // 128) * 512, dtype=torch.uint8, device=dev)
    part = torch.empty((slots, T, R), dtype=torch.float32, device=dev)
    xsd = torch.empty((T, R), dtype=torch.bfloat16, device=dev)
    _nx.call("mxm_gemm_glu", _nx.ptr(q), q.stride(0), _nx.ptr(sc), _nx.ptr(w), w.stride(0), _nx.ptr(ws), T, N, H,
             _nx.ptr(gu), _nx.ptr(xs), _nx.ptr(bg), _nx.ptr(bu), _nx.ptr(ad), R, float(s_g), float(s_u),
             _nx.ptr(qh), _nx.ptr(sh), _nx.ptr(part), _nx.ptr(xsd), _nx.stream_of(q))
    return gu, qh, sh.view(_E8), xsd


FUSE_GLU = [True]   # gate|up GEMM + forward epilogue in one kernel (rank 16); False: two passes


def _bwd_launch(gu, xs, dhm, dxd, bg, bu, ad, s_g, s_u, need_q, zero_slots=False, gu_lora=False):
    T, N2 = gu.shape
    N, R = N2 // 2, ad.shape[0]
    dev = gu.device
    sb, ncg = _nx.mlp_bwd_partitions(T, N, R)
    nsb = _cdiv(_cdiv(T, 128) * 128, sb)
    q = s = None
    if need_q:
        q = torch.empty((T, N2), dtype=_F8, device=dev)
        s = torch.empty(_cdiv(T, 128) * (N2 // 128) * 512, dtype=torch.uint8, device=dev)
    # per-row partial slots: a row block fills only the slots of the CTAs that worked on it
    dxa = (torch.zeros if zero_slots else torch.empty)((ncg, T, 3 * R), dtype=torch.float32, device=dev)
    dbg = torch.empty((nsb, N, R), dtype=torch.float32, device=dev)
    dbu = torch.empty((nsb, N, R), dtype=torch.float32, device=dev)
    dad = torch.empty((nsb, R, N), dtype=torch.float32, device=dev)
    _nx.call("mxm_mlp_bwd_epilogue", _nx.ptr(gu), _nx.ptr(xs), _nx.ptr(dhm), _nx.ptr(dxd), _nx.ptr(bg), _nx.ptr(bu),
             _nx.ptr(ad), T, N, R, float(s_g), float(s_u), int(gu_lora), _nx.ptr(q), _nx.ptr(s), _nx.ptr(dxa),
             _nx.ptr(dbg), _nx.ptr(dbu), _nx.ptr(dad), sb, ncg, _nx.stream_of(gu))
    return q, s, (dxa, dbg, dbu, dad, sb, ncg)


def mlp_bwd(gu, xs, dhm, dxd, bg, bu, ad, s_g, s_u, need_q, gu_lora=False):
    """-> (q_dgu [T, 2N] fp8, s_dgu, [dxa_gate | dxa_up | xS_down] [T, 3R] fp32 (dxa not yet scaled by s),
    dBg, dBu [N, R] fp32 (not scaled), dAd [R, N]) -- scripts/fused_mlp.py:235-259.  gu as the reference
    passes it ([x W_gate^T | x W_up^T]); gu_lora=True: gu as gemm_glu returns it (g | u, rank 16)."""
    q, s, (dxa, dbg, dbu, dad, sb, ncg) = _bwd_launch(gu, xs, dhm, dxd, bg, bu, ad, s_g, s_u, need_q, True, gu_lora)
    red = lambda p: p[0] if p.shape[0] == 1 else p.sum(0)  # noqa: E731  (fixed order on one device)
    return (q, s.view(_E8) if need_q else None, red(dxa), red(dbg), red(dbu), red(dad))


# ------------------------------------------------------------------------------------------------ autograd
class _MLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, meta, need_out, Ag, Bg, Au, Bu, Ad, Bd):
        ctx.set_materialize_grads(False)
        hold, down, (s_g, s_u, s_d), dt = meta
        lead, K = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, K)
        if x2.dtype != dt or not x2.is_contiguous():
            x2 = x2.to(dt).contiguous()
        P = _cast(("prep", id(Ag), id(Au), id(Bg), id(Bu), id(Ad), id(Bd), s_d, dt),
                  lambda: lora_prep(*(w.detach() for w in (Ag, Au, Bg, Bu, Ad, Bd)), s_d) if dt == torch.bfloat16
                  else None)
        if P is not None:
            S, bg, bu, ad, bd, bds, bdT, ST = P
        else:   # parameters in another dtype / layout: the reference's per-tensor casts
            S = _cast(((id(Ag), id(Au)), dt), lambda: torch.cat([Ag.detach().to(dt), Au.detach().to(dt)]))
            bg = _cast((id(Bg), dt), lambda: Bg.detach().to(dt).contiguous())
            bu = _cast((id(Bu), dt), lambda: Bu.detach().to(dt).contiguous())
            ad = _cast(((id(Ad),), dt), lambda: torch.cat([Ad.detach().to(dt)]))
            bd = _cast((id(Bd), dt), lambda: Bd.detach().to(dt).contiguous())
            bds = _cast(("s", id(Bd), s_d, dt), lambda: (bd.float() * s_d).to(dt).contiguous())
            bdT = _cast(("T", id(bd)), lambda: bd.t().contiguous())
            ST = _cast(("T", id(S)), lambda: S.t().contiguous())
        xs, q, sc = rowdot_quant(x2, S)                                  # [T, 2R] = xa_gate | xa_up; MXFP8(x)
        gu_lora = need_out and FUSE_GLU[0] and ad.shape[0] == 16 and hold.w.is_contiguous()
        if gu_lora:   # one pass: gu comes back as [g | u] with the LoRA terms added
            gu, qh, sh, xsd = gemm_glu(q, sc, hold.w, hold.ws, xs, bg, bu, ad, s_g, s_u)
            del q, sc
        else:
            gu = mxfp8.mx_mm(q, hold.w.t(), sc, hold.ws)                 # [T, 2N] gate | up
            del q, sc
            if need_out:
                qh, sh, xsd = mlp_fwd(gu, xs, bg, bu, ad, s_g, s_u, True)
        if need_out:
            y = mx_mm_lora(qh, down._mx_w.t(), sh, down._mx_ws, xsd, bds)
            del qh, sh, xsd
        else:   # graph only (checkpoint recompute): nobody reads the output value
            STATS["bỏ đầu ra"] = STATS.get("bỏ đầu ra", 0) + 1
            y = x2.new_empty(x2.shape[0], down.out_features)
        ctx.save_for_backward(x2, xs, gu, S, bg, bu, ad, bd)
        ctx.gu_lora = gu_lora
        ctx.meta = (hold, down, (s_g, s_u, s_d), dt, lead, K, x.dtype)
        ctx.tr = (bdT, ST)   # parameter-derived transposes (not activations)
        ctx.gdt = tuple(w.dtype for w in (Ag, Au, Bd))
        ctx.params = (Ag, Bg, Au, Bu, Ad, Bd)   # to place bucketed gradients (mx_dp.LayerGrads)
        return y.view(*lead, y.shape[-1])

    @staticmethod
    def backward(ctx, dy):
        if dy is None:
            return (None,) * 9
        x2, xs, gu, S, bg, bu, ad, bd = ctx.saved_tensors
        hold, down, (s_g, s_u, s_d), dt, lead, K, xdt = ctx.meta
        need_x = ctx.needs_input_grad[0]
        R = ad.shape[0]
        dy2 = dy.reshape(-1, dy.shape[-1]).to(dt)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        T, N = gu.shape[0], gu.shape[1] // 2
        bdT, ST = ctx.tr
        dxd, qd, sd = rowdot_quant(dy2, bdT, post=s_d)                    # bf16(bf16(dy @ Bd) * s_d); MXFP8(dy)
        wt, wts = mxfp8.mx_wt(down)
        dhm = mxfp8.mx_mm(qd, wt.t(), sd, wts)                           # [T, N]
        del qd, sd
        qg, sg, (dxa_p, dbg_p, dbu_p, dad_p, sb, ncg) = _bwd_launch(gu, xs, dhm, dxd, bg, bu, ad, s_g, s_u, need_x,
                                                                    gu_lora=ctx.gu_lora)
        del dhm
        dev = gu.device
        Ag, Bg, Au, Bu, Ad, Bd = ctx.params
        ws_in = ctx.needs_input_grad[3:]
        dst = lambda p, k: mx_dp.grad_out(p) if ws_in[k] else None  # noqa: E731  (storage of a bucketed grad)
        dxa = torch.empty((T, 2 * R), dtype=dt, device=dev)
        xsd = torch.empty((T, R), dtype=dt, device=dev)
        dB_g = _or_empty(dst(Bg, 1), (N, R), dev)
        dB_u = _or_empty(dst(Bu, 3), (N, R), dev)
        dA_d = _or_empty(dst(Ad, 4), (R, N), dev)
        _nx.call("mxm_mlp_bwd_reduce", _nx.ptr(dxa_p), _nx.ptr(dbg_p), _nx.ptr(dbu_p), _nx.ptr(dad_p), T, N, R,
                 float(s_g), float(s_u), sb, ncg, _nx.ptr(dxa), _nx.ptr(xsd), _nx.ptr(dB_g), _nx.ptr(dB_u),
                 _nx.ptr(dA_d), _nx.stream_of(gu))
        del dxa_p, dbg_p, dbu_p, dad_p
        f32 = lambda k: torch.float32 if ctx.gdt[k] == torch.float32 else torch.bfloat16  # noqa: E731
        dB_d = coldot(dy2, xsd, post=s_d, out_dtype=f32(2),              # bf16(bf16(dy^T xS_down) * s_d) [H, R]
                      out=dst(Bd, 5) if f32(2) == torch.float32 else None)
        dx = None
        if need_x:
            dx = mx_mm_lora(qg, hold.wt.t(), sg.view(_E8), hold.wts, dxa, ST)   # K = 2N: gate + up
            del qg, sg
            dx = dx.view(*lead, K).to(xdt)
        dA_dt = f32(0) if ctx.gdt[0] == ctx.gdt[1] else torch.bfloat16
        lg = mx_dp._ACTIVE[0]
        dA_out = (lg.slot_pair(Ag, Au, (2 * R, x2.shape[1]))
                  if lg is not None and dA_dt == torch.float32 and ws_in[0] and ws_in[2] else None)
        dA = coldot(x2, dxa, transpose_out=True, out_dtype=dA_dt, out=dA_out)   # [2R, H] = [dA_gate; dA_up]
        grads = [dA[:R], dB_g, dA[R:], dB_u, dA_d, dB_d]
        return (dx, None, None, *[g if ws_in[k] else None for k, g in enumerate(grads)])


def _or_empty(t, shape, dev):
    return t if t is not None else torch.empty(shape, dtype=torch.float32, device=dev)


def _r_ok(r):
    return r in (16, 32)


def mlp(mlp_mod, x, need_out=True):
    """down(silu(gate(x)) * up(x)) through _MLP when gate/up/down are PEFT LoRA layers over MX weights with
    gate/up paired (mxfp8.enable_mxfp8) and the compute dtype is bf16; otherwise None so the caller runs
    its unfused path (scripts/fused_mlp.py:343-366)."""
    if not ENABLED[0]:
        return None
    parts = [_part(m) for m in (mlp_mod.gate_proj, mlp_mod.up_proj, mlp_mod.down_proj)]
    if any(p is None or p[1] is None for p in parts):
        return None
    (gb, Ag, Bg, s_g), (ub, Au, Bu, s_u), (db, Ad, Bd, s_d) = parts
    dt = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else x.dtype
    if dt != torch.bfloat16 or not x.is_cuda:
        return None
    pg, pu = getattr(gb, "_mx_gu", None), getattr(ub, "_mx_gu", None)
    if pg is None or pu is None or pg[0] is not pu[0] or (pg[1], pu[1]) != (0, 1) or not mxfp8.is_mx(db):
        return None
    hold = pg[0]
    r = Ag.shape[0]
    T = x.numel() // x.shape[-1]
    if not (_r_ok(r) and Au.shape[0] == r and Ad.shape[0] == r and x.shape[-1] == hold.w.shape[1]
            and hold.n % 128 == 0 and Ad.shape[1] == hold.n and T > 0 and T * 2 * hold.n < 2 ** 31):
        return None
    STATS["mlp gộp"] = STATS.get("mlp gộp", 0) + 1
    ACTIVE[0] = True
    return _MLP.apply(x, (hold, db, (s_g, s_u, s_d), dt), need_out, Ag, Bg, Au, Bu, Ad, Bd)


# ------------------------------------------------------------------------------------------------ standalone use
class MXMLPWeights:
    """Frozen MLP weights in the layout ``mxfp8.enable_mxfp8`` builds for one layer: ``hold`` (the shared
    gate|up codes in both orientations) and ``down`` (W_down codes in both orientations).  For callers that
    drive ``_MLP`` without a PEFT model (benchmarks, tests)."""

    def __init__(self, hold, down):
        self.hold, self.down = hold, down

    @classmethod
    def from_bf16(cls, w_gate, w_up, w_down):
        w = torch.cat([w_gate, w_up]).to(torch.bfloat16).contiguous()
        n = w_gate.shape[0]
        hold = types.SimpleNamespace(n=n, half_t=[None, None])
        hold.w, hold.ws, hold.wt, hold.wts = mxfp8.mx_quant_pair(w)
        down = types.SimpleNamespace(out_features=w_down.shape[0])
        down._mx_w, down._mx_ws, down._mx_wt, down._mx_wts = mxfp8.mx_quant_pair(w_down.to(torch.bfloat16).contiguous())
        return cls(hold, down)


def mlp_apply(layer, x, Ag, Bg, Au, Bu, Ad, Bd, scaling=(1.0, 1.0, 1.0), need_out=True):
    """_MLP.apply on explicit weights: y = down(silu(gate(x)) * up(x)) with LoRA on all three projections."""
    return _MLP.apply(x, (layer.hold, layer.down, tuple(float(s) for s in scaling), torch.bfloat16), need_out,
                      Ag, Bg, Au, Bu, Ad, Bd)
