"""Linears that share one input, computed in ONE autograd node on the B200 kernels: drop-in for the
reference module of the same name (scripts/fused_linear.py).  Public surface kept: ``group_linear``,
``residual_add``, ``Deferred``, ``_part``, ``_cast`` / ``new_step`` and ``STATS`` (``fused_mlp`` imports
the last three, scripts/fused_mlp.py:27; ``shared_prefix`` calls the first ones).

A call ``group_linear(x, mods)`` is described by a ``_Layout``: the columns of the skinny matrix S
(every LoRA A of the group, then the weights of thin frozen linears of <= 64 outputs) and, per output,
whether its frozen weight is MXFP8 (``mxfp8.enable_mxfp8``).  Forward: x S^T once for the whole group
(tensor-core rowdot), x quantized once for every MX output, each MX output one tcgen05 GEMM with its LoRA
term accumulated in the same accumulator (or left to ``residual_add`` when deferred).  Backward, when the
whole group is MX and bf16 (``_one_read_plan``): ONE native call (``mxm_group_lora_bwd``) reads each dy
once for its MXFP8 codes (into the group's K-concatenated operand), its d(xa) and its dB; the group's
dx is ONE MXFP8 GEMM against the concatenated W^T with dS S accumulated inside it, and dA = dS^T x one
coldot.  Any other group (fp32, bf16 weights, a missing output gradient, a rank the kernels do not
take) runs the general path, with the reference's arithmetic.
"""
import collections

import torch
from torch import nn

_THIN = 64
STATS = {"gộp": 0, "gọi thẳng": 0}


def _bump(key):
    STATS[key] = STATS.get(key, 0) + 1


def _part(m):
    """(base Linear, A, B, scaling) of a PEFT LoRA Linear, (m, None, None, 1.0) for a plain frozen Linear,
    None when the layer cannot take the grouped path: trainable or biased base, merged / disabled adapters,
    several active adapters, DoRA or another variant, a LoRA bias, dropout (scripts/fused_linear.py:30-48)."""
    base = getattr(m, "base_layer", None)
    if base is None:
        plain = type(m) is nn.Linear and m.bias is None and not m.weight.requires_grad
        return (m, None, None, 1.0) if plain else None
    if base.bias is not None or base.weight.requires_grad or m.merged or m.disable_adapters:
        return None
    active = [a for a in m.active_adapters if a in m.lora_A]
    if len(active) != 1:
        return None
    a = active[0]
    drop = m.lora_dropout[a]
    no_drop = isinstance(drop, nn.Identity) or getattr(drop, "p", 1) == 0
    if a in getattr(m, "lora_variant", {}) or m.use_dora.get(a, False) or m.lora_B[a].bias is not None or not no_drop:
        return None
    return base, m.lora_A[a].weight, m.lora_B[a].weight, m.scaling[a]


def _is_mx(base):
    return getattr(base, "_mx_w", None) is not None


# Per-step cache of derived LoRA tensors (bf16 casts, concatenations, transposes).  Optimizers update the
# parameters in place without bumping their version counter, so entries are keyed by parameter identity
# and the whole cache is dropped by new_step() at the start of every step (scripts/fused_linear.py:55-69).
_CAST = {}


def new_step():
    _CAST.clear()


def _cast(key, make):
    hit = _CAST.get(key)
    if hit is None:
        hit = _CAST[key] = make()
    return hit


def _compute_dtype(x):
    return torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else x.dtype


Branch = collections.namedtuple("Branch", "out col rank scale")   # a LoRA branch: output, S column, r, s
Thin = collections.namedtuple("Thin", "out col width")            # a thin frozen linear inside S


class _Layout:
    """Column layout of one group call.  S rows: the LoRA A's in output order, then thin frozen weights."""

    def __init__(self, parts):
        self.parts = parts
        self.branches, self.thin, col = [], [], 0
        for i, (base, A, B, s) in enumerate(parts):
            if A is not None:
                self.branches.append(Branch(i, col, A.shape[0], s))
                col += A.shape[0]
        self.lora_width = col
        for i, (base, A, B, s) in enumerate(parts):
            if A is None and not _is_mx(base) and base.weight.shape[0] <= _THIN:
                self.thin.append(Thin(i, col, base.weight.shape[0]))
                col += base.weight.shape[0]
        self.width = col
        self.thin_outs = {t.out for t in self.thin}
        self.by_out = {b.out: b for b in self.branches}
        self.mx = [i for i, p in enumerate(parts) if _is_mx(p[0])]

    def s_rows(self):
        return [self.parts[b.out][1] for b in self.branches] + [self.parts[t.out][0].weight for t in self.thin]


def _rowdot_ok(x2, S):
    return (x2.dtype == S.dtype == torch.bfloat16 and S.shape[0] in (16, 32, 64) and x2.shape[1] % 128 == 0
            and x2.is_contiguous())


def _skinny(x2, S):
    """x2 @ S^T: the tensor-core rowdot for 16 / 32 / 64 bf16 columns, a plain matmul otherwise."""
    if _rowdot_ok(x2, S):
        import fused_mlp
        return fused_mlp.rowdot(x2, S)
    return x2 @ S.t()


class _GroupFn(torch.autograd.Function):
    """The group as one autograd node (scripts/fused_linear.py:79-196).  Inputs after `defer`: (A, B) of
    every LoRA branch in output order."""

    @staticmethod
    def forward(ctx, x, lay, need_out, defer, *ws):
        ctx.set_materialize_grads(False)   # an output nobody uses gets a None gradient, not zeros
        dt = _compute_dtype(x)
        lead, K = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, K)
        if x2.dtype != dt or not x2.is_contiguous():
            x2 = x2.to(dt).contiguous()
        rows = lay.s_rows()
        S = _cast(("S", tuple(id(r) for r in rows), dt), lambda: torch.cat([r.detach().to(dt) for r in rows])) \
            if rows else None
        Bs = [_cast((id(lay.parts[b.out][2]), dt), lambda b=b: lay.parts[b.out][2].detach().to(dt).contiguous())
              for b in lay.branches]
        xS = _skinny(x2, S) if S is not None else None
        outs = [None] * len(lay.parts)
        if need_out:
            _forward_outputs(lay, x2, xS, Bs, dt, defer, outs)
        else:   # graph only (checkpoint recompute): nothing reads the outputs, the backward needs x2 and xS
            _bump("bỏ đầu ra")
            for i, (base, A, B, s) in enumerate(lay.parts):
                if i not in lay.thin_outs:
                    outs[i] = x2.new_empty(x2.shape[0], base.out_features)
        for t in lay.thin:
            outs[t.out] = xS[:, t.col:t.col + t.width].contiguous()
        ctx.save_for_backward(x2, xS, S, *Bs)
        ctx.lay, ctx.shape, ctx.dt = lay, (lead, K, x.dtype), dt
        return tuple(y.view(*lead, y.shape[-1]) for y in outs)

    @staticmethod
    def backward(ctx, *dys):
        x2, xS, S, *Bs = ctx.saved_tensors
        lay, dt = ctx.lay, ctx.dt
        need_x = ctx.needs_input_grad[0]
        flat = [None if dy is None else dy.reshape(-1, dy.shape[-1]).to(dt) for dy in dys]
        plan = _one_read_plan(lay, flat, dt, need_x, xS, Bs)
        if plan is not None:
            dx, grads = _backward_one_read(lay, x2, xS, S, Bs, flat, plan, need_x)
            _bump("lan ngược gộp")
        else:
            dx, grads = _backward_general(lay, x2, xS, S, Bs, flat, dt, need_x)
        lead, K, xdt = ctx.shape
        keep = ctx.needs_input_grad[4:]
        grads = [g if (g is not None and keep[k]) else None for k, g in enumerate(grads)]
        return (None if dx is None else dx.view(*lead, K).to(xdt), None, None, None, *grads)


def _forward_outputs(lay, x2, xS, Bs, dt, defer, outs):
    """Frozen-weight products of the non-thin outputs with their LoRA terms: MX outputs on the tcgen05 GEMM
    (x quantized once for the group), bf16 ones with a matmul."""
    import mxfp8
    qx = mxfp8.mx_quant(x2) if lay.mx else None
    for i, (base, A, B, s) in enumerate(lay.parts):
        if i in lay.thin_outs:
            continue
        br = lay.by_out.get(i)
        xa = None if br is None else xS[:, br.col:br.col + br.rank]
        j = None if br is None else lay.branches.index(br)
        if _is_mx(base):
            if br is not None and defer is not None and dt == torch.bfloat16:
                outs[i] = mxfp8.mx_mm(qx[0], base._mx_w.t(), qx[1], base._mx_ws)
                defer[i] = (xa, Bs[j], s)          # residual_add adds the LoRA term in its kernel
                continue
            if br is not None:
                Bsc = _cast(("scaled", id(B), s, dt), lambda: (Bs[j].float() * s).to(dt).contiguous())
                if mxfp8.mx_mm_lora_ok(xa, Bsc):
                    outs[i] = mxfp8.mx_mm_lora(qx[0], base._mx_w.t(), qx[1], base._mx_ws, xa, Bsc)
                    continue
            outs[i] = mxfp8.mx_mm(qx[0], base._mx_w.t(), qx[1], base._mx_ws)
        else:
            outs[i] = x2 @ base.weight.to(dt).t()
        if br is not None:
            outs[i].addmm_(xa, Bs[j].t(), alpha=s)


# ------------------------------------------------------------------------------------------------ backward
def _one_read_plan(lay, flat, dt, need_x, xS, Bs):
    """The one-read backward applies when the compute dtype is bf16, every output has a gradient, every MX
    output was marked for it by enable_mxfp8 (mxfp8.FUSED_BWD), the group's MX weights form one
    concatenated W^T in output order (when dx is needed), every bf16-base LoRA branch is absent and the
    kernels take every branch (scripts/fused_linear.py:203-216).  Returns the W^T operand (or True when dx
    is not needed), else None."""
    import mxfp8
    if dt != torch.bfloat16 or any(d is None for d in flat) or not lay.mx:
        return None
    if not all(getattr(lay.parts[i][0], "_mx_fbwd", False) for i in lay.mx):
        return None
    if any(not _is_mx(lay.parts[b.out][0]) for b in lay.branches):
        return None
    for i in lay.mx:
        br = lay.by_out.get(i)
        if not mxfp8.lora_bwd_ok(flat[i], None if br is None else xS[:, br.col:br.col + br.rank], None
                                 if br is None else Bs[lay.branches.index(br)]):
            return None
    if not need_x:
        return True
    return mxfp8.group_wt([lay.parts[i][0] for i in lay.mx])


def _backward_one_read(lay, x2, xS, S, Bs, flat, wt, need_x):
    """(scripts/fused_linear.py:219-278): per MX output one read of dy in ONE native call, then dx as ONE
    MX GEMM with dS S accumulated inside it and dA = dS^T x2."""
    import fused_mlp
    import mxfp8
    T, dev, dt = x2.shape[0], x2.device, x2.dtype
    dS = torch.empty((T, lay.width), dtype=dt, device=dev) if lay.width else None
    grads = [None] * (2 * len(lay.branches))
    q = s = None
    if need_x:
        n_mx = sum(flat[i].shape[1] for i in lay.mx)
        q = torch.empty((T, n_mx), dtype=mxfp8.F8, device=dev)
        s = torch.empty(mxfp8.scale_numel(T, n_mx), dtype=torch.uint8, device=dev)
    work = []
    for i in lay.mx:
        dy = flat[i] if flat[i].stride(1) == 1 else flat[i].contiguous()
        flat[i] = dy
        br = lay.by_out.get(i)
        if br is None:
            work.append((dy, None, None, 0.0, None, None))
            continue
        j = lay.branches.index(br)
        Bt = _cast(("T", id(lay.parts[i][2]), dt), lambda j=j: Bs[j].t().contiguous())
        grads[2 * j + 1] = torch.empty((dy.shape[1], br.rank), dtype=torch.float32, device=dev)
        work.append((dy, xS[:, br.col:br.col + br.rank], Bt, br.scale, dS[:, br.col:br.col + br.rank],
                     grads[2 * j + 1]))
    if q is None:   # no dx: only the LoRA branches have work
        work = [w for w in work if w[1] is not None]
    if work:
        mxfp8.group_lora_bwd(T, work, q, s, device=dev)
    dx = None
    if need_x:
        for t in lay.thin:
            dS[:, t.col:t.col + t.width].copy_(flat[t.out])
        sv = s.view(mxfp8.E8)
        ST = _cast(("ST", id(S)), lambda: S.t().contiguous()) if S is not None else None
        if dS is not None and mxfp8.mx_mm_lora_ok(dS, ST):
            dx = mxfp8.mx_mm_lora(q, wt[0], sv, wt[1], dS, ST)            # dy W (all MX outputs) + dS S
        else:
            dx = mxfp8.mx_mm(q, wt[0], sv, wt[1])
            if dS is not None:
                dx.addmm_(dS, S)
        del q, s
        for i, (base, A, B, sc) in enumerate(lay.parts):                  # plain bf16 linears, if any
            if i not in lay.thin_outs and not _is_mx(base):
                dx.addmm_(flat[i], base.weight.to(dt))
    if lay.branches:
        n = lay.lora_width
        if n in (16, 32, 64) and x2.shape[1] % 64 == 0:
            dA = fused_mlp.coldot(x2, dS[:, :n], transpose_out=True)     # [n, K] = dS^T x2
        else:
            dA = dS[:, :n].t() @ x2
        for j, br in enumerate(lay.branches):
            grads[2 * j] = dA[br.col:br.col + br.rank]
    return dx, grads


def _backward_general(lay, x2, xS, S, Bs, flat, dt, need_x):
    """The general path (scripts/fused_linear.py:132-196): frozen-weight dx per output (MX outputs through
    MXFP8(dy) and their own W^T), LoRA dB / d(xa) per branch, thin linears' dy as columns of dS, then
    dx += dS S and dA = dS^T x2 for the branches that got a gradient."""
    import mxfp8
    dx = None
    if need_x:
        for i, (base, A, B, s) in enumerate(lay.parts):
            dy = flat[i]
            if dy is None or i in lay.thin_outs:
                continue
            if _is_mx(base):
                d = dy if dy.is_contiguous() else dy.contiguous()
                qd, sd = mxfp8.mx_quant(d)
                mat2, ws = mxfp8.wt_of(base)
                g = mxfp8.mx_mm(qd, mat2, sd, ws)
                dx = g if dx is None else dx.add_(g)
            else:
                w = base.weight.to(dt)
                dx = dy @ w if dx is None else dx.addmm_(dy, w)
    grads = [None] * (2 * len(lay.branches))
    cols, srows, live = [], [], []
    for j, br in enumerate(lay.branches):
        dy = flat[br.out]
        if dy is None:
            continue
        xa = xS[:, br.col:br.col + br.rank]
        dB, dxa = dy.t() @ xa, dy @ Bs[j]
        if br.scale != 1:
            dB.mul_(br.scale)
            dxa.mul_(br.scale)
        grads[2 * j + 1] = dB
        cols.append(dxa)
        srows.append((br.col, br.rank))
        live.append(j)
    n_live = sum(w for _, w in srows)
    if need_x:
        for t in lay.thin:
            if flat[t.out] is not None:
                cols.append(flat[t.out])
                srows.append((t.col, t.width))
    if cols:
        dS = torch.cat(cols, 1) if len(cols) > 1 else cols[0]
        if need_x:
            Sa = S if sum(w for _, w in srows) == lay.width else torch.cat([S[c:c + w] for c, w in srows])
            dx = dS @ Sa if dx is None else dx.addmm_(dS, Sa)
        if live:
            dA = dS[:, :n_live].t() @ x2
            c = 0
            for j in live:
                r = lay.branches[j].rank
                grads[2 * j] = dA[c:c + r]
                c += r
    return dx, grads


# ------------------------------------------------------------------------------------------------ residual + LoRA
class Deferred(tuple):
    """(y, xa, B, scaling): the MX bf16 output of o_proj / out_proj without its LoRA term, which
    residual_add adds inside the residual kernel (scripts/fused_linear.py:282-283)."""


class _ResidualAdd(torch.autograd.Function):
    """x + (y + s * xa @ B^T) in one kernel (scripts/fused_linear.py:286-299).  xa and B arrive detached: the
    LoRA branch's gradients come from the group's backward (same dy), so this node passes dy to x and y."""

    @staticmethod
    def forward(ctx, x, y, xa, B, s):
        import mxfp8
        N = x.shape[-1]
        return mxfp8.res_lora(x.reshape(-1, N), y.reshape(-1, N), xa, B, s).view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        return dy, dy, None, None, None


def residual_add(x, y):
    """x + y; when y is a Deferred (group_linear(..., defer=True)) its LoRA term is added inside the
    residual kernel (scripts/fused_linear.py:302-312), or by an addmm where the kernel does not apply."""
    if not isinstance(y, Deferred):
        return x + y
    import mxfp8
    y, xa, B, s = y
    N = x.shape[-1]
    if x.shape == y.shape and mxfp8.res_lora_ok(x.reshape(-1, N), y.reshape(-1, N), xa, B):
        _bump("residual LoRA")
        return _ResidualAdd.apply(x, y, xa, B, s)
    return x + torch.addmm(y.reshape(-1, N), xa, B.t(), alpha=s).view(y.shape)


def group_linear(x, mods, need_out=True, defer=False):
    """(m(x) for m in mods) through one node (scripts/fused_linear.py:315-335).  need_out=False builds only
    the graph for backward (outputs uninitialized, gradients unchanged) -- the last layer of a checkpointed
    segment being recomputed.  defer=True returns the MX bf16 outputs that carry a LoRA branch as Deferred,
    for a residual_add that follows right away."""
    parts = tuple(_part(m) for m in mods)
    if any(p is None for p in parts):
        STATS["gọi thẳng"] += 1
        return tuple(m(x) for m in mods)
    STATS["gộp"] += 1
    lay = _Layout(parts)
    ws = [w for b in lay.branches for w in (parts[b.out][1], parts[b.out][2])]
    box = {} if defer and need_out else None
    outs = _GroupFn.apply(x, lay, need_out, box, *ws)
    if not box:
        return outs
    return tuple(Deferred((y,) + box[i]) if i in box else y for i, y in enumerate(outs))
