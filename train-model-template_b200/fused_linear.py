"""Linears that share one input computed in ONE autograd node, on the B200 kernels: drop-in for the
reference module of the same name (scripts/fused_linear.py).

* ``group_linear(x, mods, need_out, defer)`` -- q/k/v, qkv/z/b/a, o_proj ... as one node: x read once for all
  LoRA A's, one MXFP8 quantization of x for the group, LoRA gradients into dx through one addmm; on the
  MX path the backward reads each dy once (``mxfp8.lora_bwd``) and computes the group's dx as one MXFP8
  GEMM against the concatenated W^T.
* ``residual_add(x, y)`` -- the residual add, with the deferred LoRA term of o_proj / out_proj added in the
  same kernel (``mxfp8.res_lora``).
* ``_part``, ``_cast`` / ``new_step``, ``STATS`` -- the LoRA-layer decomposition, the per-step bf16 cast cache
  and the path counters that ``fused_mlp`` imports (scripts/fused_mlp.py:27) and ``shared_prefix`` uses.
"""
import torch
from torch import nn

_THIN = 64
STATS = {"gộp": 0, "gọi thẳng": 0}


def _part(m):
    """(base Linear, A, B, scaling) of a PEFT LoRA Linear, (m, None, None, 1.0) for a plain frozen Linear,
    None when the layer cannot take the fused path (scripts/fused_linear.py:30-48)."""
    base = getattr(m, "base_layer", None)
    if base is None:
        if type(m) is nn.Linear and m.bias is None and not m.weight.requires_grad:
            return m, None, None, 1.0
        return None
    if base.bias is not None or base.weight.requires_grad or m.merged or m.disable_adapters:
        return None
    ads = [a for a in m.active_adapters if a in m.lora_A]
    if len(ads) != 1:
        return None
    a = ads[0]
    drop = m.lora_dropout[a]
    if (a in getattr(m, "lora_variant", {}) or m.use_dora.get(a, False) or m.lora_B[a].bias is not None
            or not (isinstance(drop, nn.Identity) or getattr(drop, "p", 1) == 0)):
        return None
    return base, m.lora_A[a].weight, m.lora_B[a].weight, m.scaling[a]


def _mx(base):
    return getattr(base, "_mx_w", None) is not None


# bf16 copies of the LoRA parameters, made once per step (scripts/fused_linear.py:55-69).  The
# optimizer updates parameters in place without bumping _version, so the cache is keyed by id and
# cleared by new_step() at the start of each step.
_CAST = {}


def new_step():
    _CAST.clear()


def _cast(key, make):
    t = _CAST.get(key)
    if t is None:
        t = _CAST[key] = make()
    return t


# ------------------------------------------------------------------------------------------------ grouped linears
def _base_mm(base, x2, dt, q):
    """x2 @ W^T of a frozen base linear: the MXFP8 GEMM when enable_mxfp8 quantized it (q = MXFP8(x2)),
    a plain matmul otherwise (scripts/fused_linear.py:72-76)."""
    if _mx(base):
        import mxfp8
        return mxfp8.mx_mm(q[0], base._mx_w.t(), q[1], base._mx_ws)
    return x2 @ base.weight.to(dt).t()


def _compute_dtype(x):
    return torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else x.dtype


class _Group(torch.autograd.Function):
    """Linears that share one input (q/k/v, qkv/z/b/a, gate/up, o_proj alone ...) as one autograd node
    (scripts/fused_linear.py:79-196).  x is read once for every LoRA A of the group and for the weights of
    thin frozen linears (<= _THIN outputs), stacked as the rows of one matrix S; the gradients of all
    LoRA branches and thin linears reach dx through one addmm with S; dA for every branch is one GEMM.
    Inputs after `defer`: (A, B) of each LoRA branch in group order."""

    @staticmethod
    def forward(ctx, x, parts, need_out, defer, *ws):
        ctx.set_materialize_grads(False)   # an unused output gives a None gradient, not zeros
        dt = _compute_dtype(x)
        lead, K = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, K)
        if x2.dtype != dt or not x2.is_contiguous():
            x2 = x2.to(dt).contiguous()
        srows, Bs, lora, thin = [], [], [], []   # rows of S; bf16 B's; (part, row offset, rank, s); (part, offset, n)
        for i, (base, A, B, s) in enumerate(parts):
            if A is not None:
                lora.append((i, sum(r.shape[0] for r in srows), A.shape[0], s))
                srows.append(A)
                Bs.append(_cast((id(B), dt), lambda B=B: B.detach().to(dt)))
        for i, (base, A, B, s) in enumerate(parts):
            if A is None and not _mx(base) and base.weight.shape[0] <= _THIN:
                thin.append((i, sum(r.shape[0] for r in srows), base.weight.shape[0]))
                srows.append(base.weight)
        S = None
        if srows:
            S = _cast((tuple(id(r) for r in srows), dt), lambda: torch.cat([r.detach().to(dt) for r in srows]))
        xS = x2 @ S.t() if S is not None else None
        thin_idx = {i for i, _, _ in thin}
        outs = [None] * len(parts)
        if need_out:
            q = None
            if any(_mx(p[0]) for p in parts):
                import mxfp8
                q = mxfp8.mx_quant(x2)           # one quantization for the whole group
            for i, (base, A, B, s) in enumerate(parts):
                if i not in thin_idx:
                    outs[i] = _base_mm(base, x2, dt, q)
            for j, (i, o, r, s) in enumerate(lora):
                if defer is not None and _mx(parts[i][0]) and dt == torch.bfloat16:
                    defer[i] = (xS[:, o:o + r], Bs[j], s)   # added by residual_add inside the residual kernel
                else:
                    outs[i].addmm_(xS[:, o:o + r], Bs[j].t(), alpha=s)
        else:   # graph only (checkpoint recompute): x2 and xS are saved, nobody reads the outputs
            STATS["bỏ đầu ra"] = STATS.get("bỏ đầu ra", 0) + 1
            for i, (base, A, B, s) in enumerate(parts):
                if i not in thin_idx:
                    outs[i] = x2.new_empty(x2.shape[0], base.out_features)
        for i, o, n in thin:
            outs[i] = xS[:, o:o + n].contiguous()
        ctx.save_for_backward(x2, xS, S, *Bs)
        ctx.meta = (parts, lora, thin, lead, K, dt, x.dtype)
        return tuple(y.view(*lead, y.shape[-1]) for y in outs)

    @staticmethod
    def backward(ctx, *dys):
        x2, xS, S, *Bs = ctx.saved_tensors
        parts, lora, thin, lead, K, dt, xdt = ctx.meta
        need_x = ctx.needs_input_grad[0]
        flat = [None if dy is None else dy.reshape(-1, dy.shape[-1]).to(dt) for dy in dys]
        plan = _fused_bwd_plan(parts, flat, dt, need_x)
        if plan is not None:
            return _fused_backward(ctx, x2, xS, S, Bs, flat, plan, need_x)
        # the general path (scripts/fused_linear.py:132-196)
        thin_idx = {i for i, _, _ in thin}
        dx = None
        if need_x:
            for i, (base, A, B, s) in enumerate(parts):
                dy = flat[i]
                if dy is None or i in thin_idx:
                    continue
                if _mx(base):
                    import mxfp8
                    d = dy if dy.is_contiguous() else dy.contiguous()
                    qd, sd = mxfp8.mx_quant(d)
                    wt, wts = mxfp8.wt_of(base)
                    g = mxfp8.mx_mm(qd, wt, sd, wts)
                    dx = g if dx is None else dx.add_(g)
                else:
                    w = base.weight.to(dt)
                    dx = dy @ w if dx is None else dx.addmm_(dy, w)
        grads = [None] * (2 * len(lora))
        cols, col_rows, live = [], [], []        # columns of dS, the S rows they multiply, active branches
        for j, (i, o, r, s) in enumerate(lora):
            dy = flat[i]
            if dy is None:
                continue
            xa = xS[:, o:o + r]
            dB, dxa = dy.t() @ xa, dy @ Bs[j]
            if s != 1:
                dB.mul_(s)
                dxa.mul_(s)
            grads[2 * j + 1] = dB
            cols.append(dxa)
            col_rows.append((o, r))
            live.append(j)
        n_live = sum(r for _, r in col_rows)
        if need_x:
            for i, o, n in thin:
                if flat[i] is not None:
                    cols.append(flat[i])
                    col_rows.append((o, n))
        if cols:
            dS = torch.cat(cols, 1) if len(cols) > 1 else cols[0]
            if need_x:
                Sa = S if len(col_rows) == len(lora) + len(thin) else torch.cat([S[o:o + n] for o, n in col_rows])
                dx = dS @ Sa if dx is None else dx.addmm_(dS, Sa)
            if live:
                dA = dS[:, :n_live].t() @ x2
                c = 0
                for j in live:
                    r = lora[j][2]
                    grads[2 * j] = dA[c:c + r]
                    c += r
        return _grads_out(ctx, dx, grads, lead, K, xdt)


def _grads_out(ctx, dx, grads, lead, K, xdt):
    ws_in = ctx.needs_input_grad[4:]
    out = [None if (g is None or not ws_in[k]) else g for k, g in enumerate(grads)]
    dx = None if dx is None else dx.view(*lead, K).to(xdt)
    return (dx, None, None, None, *out)


def _cdiv(a, b):
    return -(-a // b)


def _fused_bwd_plan(parts, flat, dt, need_x):
    """The one-read backward applies when the compute dtype is bf16, every output has a gradient, every MX
    branch is one enable_mxfp8 marked for it (mxfp8.FUSED_BWD) and, when dx is needed, the group's MX
    weights form one concatenated W^T in group order: returns (MX branch indices, (mat2, scales) or None),
    else None (scripts/fused_linear.py:203-216)."""
    if dt != torch.bfloat16 or any(dy is None for dy in flat):
        return None
    mx_idx = [i for i, p in enumerate(parts) if _mx(p[0])]
    if not mx_idx or not all(getattr(parts[i][0], "_mx_fbwd", False) for i in mx_idx):
        return None
    import mxfp8
    wt = mxfp8.group_wt([parts[i][0] for i in mx_idx]) if need_x else None
    if need_x and wt is None:
        return None
    return mx_idx, wt


def _fused_backward(ctx, x2, xS, S, Bs, flat, plan, need_x):
    """_Group.backward on the one-read path (scripts/fused_linear.py:219-278): each MX branch's dy is read once
    by mxfp8.lora_bwd (its MXFP8 into one K-concatenated buffer, its d(xa) into dS, its dB), and the
    group's dx is ONE MXFP8 GEMM against the concatenated W^T (the branches add in fp32 inside it), plus
    the bf16 branches and dS @ S."""
    import mxfp8
    parts, lora, thin, lead, K, dt, xdt = ctx.meta
    mx_idx, wt = plan
    T, dev = x2.shape[0], x2.device
    branch = {i: (j, o, r, s) for j, (i, o, r, s) in enumerate(lora)}
    n_lora = sum(r for _, _, r, _ in lora)
    width = n_lora + (sum(n for _, _, n in thin) if need_x else 0)
    dS = torch.empty((T, width), dtype=dt, device=dev) if width else None
    grads = [None] * (2 * len(lora))
    q = sbuf = None
    if need_x:
        n_mx = sum(flat[i].shape[1] for i in mx_idx)
        q = torch.empty((T, n_mx), dtype=mxfp8.F8, device=dev)
        sbuf = torch.empty(_cdiv(T, 128) * (n_mx // 128) * 512, dtype=torch.uint8, device=dev)
    tile = 0
    for i in mx_idx:
        dy = flat[i] if flat[i].stride(1) == 1 else flat[i].contiguous()
        if i in branch:
            j, o, r, s = branch[i]
            grads[2 * j + 1] = mxfp8.lora_bwd(dy, xS[:, o:o + r], Bs[j], s, q=q, s=sbuf, col_tile_off=tile,
                                              dxa_out=dS[:, o:o + r])
        elif need_x:
            mxfp8.lora_bwd(dy, q=q, s=sbuf, col_tile_off=tile)
        tile += dy.shape[1] // 128
    for j, (i, o, r, s) in enumerate(lora):   # LoRA over a bf16 (non-MX) base: as on the general path
        if i in mx_idx:
            continue
        dy = flat[i]
        dB = dy.t() @ xS[:, o:o + r]
        dS[:, o:o + r] = dy @ Bs[j]
        if s != 1:
            dB.mul_(s)
            dS[:, o:o + r].mul_(s)
        grads[2 * j + 1] = dB
    dx = None
    if need_x:
        dx = mxfp8.mx_mm(q, wt[0], sbuf.view(mxfp8.E8), wt[1])
        del q, sbuf
        thin_idx = {i for i, _, _ in thin}
        for i, (base, A, B, s) in enumerate(parts):   # plain bf16 linears (neither MX nor thin)
            if i not in thin_idx and not _mx(base):
                dx.addmm_(flat[i], base.weight.to(dt))
        for i, o, n in thin:
            dS[:, o:o + n].copy_(flat[i])
        if dS is not None:
            dx.addmm_(dS, S)
    if lora:
        dA = dS[:, :n_lora].t() @ x2
        for j, (i, o, r, s) in enumerate(lora):
            grads[2 * j] = dA[o:o + r]
    STATS["lan ngược gộp"] = STATS.get("lan ngược gộp", 0) + 1
    return _grads_out(ctx, dx, grads, lead, K, xdt)


# ------------------------------------------------------------------------------------------------ residual + LoRA
class Deferred(tuple):
    """(y, xa, B, scaling): the MX bf16 output of o_proj / out_proj without its LoRA term, which
    residual_add adds inside the residual kernel (scripts/fused_linear.py:282-283)."""


class _ResidualLoRA(torch.autograd.Function):
    """x + (y + s * xa @ B^T) in one kernel (scripts/fused_linear.py:286-299).  xa and B come detached: the
    LoRA branch's gradients (dB, d(xa) -> dA, dx) are produced by _Group.backward from the same dy, so
    this node only passes dy through to x and y."""

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
    residual kernel (scripts/fused_linear.py:302-312)."""
    if not isinstance(y, Deferred):
        return x + y
    y, xa, B, s = y
    N = x.shape[-1]
    if (x.dtype == y.dtype == torch.bfloat16 and x.shape == y.shape and x.is_contiguous() and y.is_contiguous()
            and N % 128 == 0 and xa.stride(1) == 1 and B.is_contiguous()):
        STATS["residual LoRA"] = STATS.get("residual LoRA", 0) + 1
        return _ResidualLoRA.apply(x, y, xa, B, s)
    return x + torch.addmm(y.reshape(-1, N), xa, B.t(), alpha=s).view(y.shape)


def group_linear(x, mods, need_out=True, defer=False):
    """(m(x) for m in mods) with the grouping above (scripts/fused_linear.py:315-335).  need_out=False builds
    only the graph for backward (the outputs are uninitialized; gradients are unchanged) -- the last
    layer of a checkpointed segment being recomputed.  defer=True returns the MX bf16 outputs that carry
    a LoRA branch as Deferred, for a residual_add that follows right away."""
    parts = tuple(_part(m) for m in mods)
    if any(p is None for p in parts):
        STATS["gọi thẳng"] += 1
        return tuple(m(x) for m in mods)
    STATS["gộp"] += 1
    ws = [w for p in parts if p[1] is not None for w in (p[1], p[2])]
    box = {} if defer and need_out else None
    outs = _Group.apply(x, parts, need_out, box, *ws)
    if not box:
        return outs
    return tuple(Deferred((y,) + box[i]) if i in box else y for i, y in enumerate(outs))
