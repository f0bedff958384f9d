"""MXFP8 (E4M3 codes, one E8M0 scale per 32 elements) for the FROZEN base weights of LoRA layers,
on B200 (sm_100a) kernels.  Drop-in for the reference module of the same name
(scripts/mxfp8.py): same public names, arguments, outputs and error behaviour.

* ``mx_quant(x2d)`` -- row-wise activation quantizer (scripts/mxfp8.py:78-86), CUDA kernel
  ``mxm_quant_rows``; codes and scales are bit-identical to the reference ``_quant_kernel``.
* ``quant_ref(x2d)`` -- the weight quantizer (scripts/mxfp8.py:40-43).  The reference computes it
  with torchao ``to_mx(..., RCEIL)`` + ``to_blocked``, which it states is identical to
  ``mx_quant`` (scripts/mxfp8.py:11); here it is the same CUDA quantizer.
* ``mx_quant_t(x2d)`` / ``mx_quant_pair(x2d)`` -- column-wise (= ``quant_ref(x.t().contiguous())``)
  and both orientations from one read, used for the weights by ``enable_mxfp8``.
* ``mx_mm(a, b, scale_a, scale_b)`` -- the MXFP8 GEMM with ``torch._scaled_mm``'s calling convention
  (``b`` is the ``.t()`` view of a [N, K] code matrix), on the tcgen05 block-scaled MMA; ``mx_mm_lora``
  adds a rank-r LoRA term inside the same accumulator.
* ``enable_mxfp8`` / ``disable_mxfp8`` / ``is_mx`` / ``mx_wt`` / ``wt_of`` / ``group_wt`` -- the frozen
  weight layouts (scripts/mxfp8.py:398-509), including the shared gate|up pair that ``fused_mlp``
  consumes.  ``enable_mxfp8`` first plans every layout the model needs, then builds them.
* ``lora_bwd`` / ``res_lora`` -- the LoRA backward of an MX linear from one read of dy (MXFP8 of dy into a
  K-concatenated buffer + d(xa) + dB) and the residual add with the LoRA term
  (scripts/mxfp8.py:88-296).  Requests the kernels do not take raise ``MXError`` with status
  ``MXM_ERR_UNSUPPORTED``; callers check ``lora_bwd_ok`` / ``res_lora_ok`` first.
"""
import os
import types
import weakref

import torch

import _mxlib as _nx

F8, E8 = torch.float8_e4m3fn, torch.float8_e8m0fnu
STATS = {"quant": 0, "reuse": 0}
MXM_ERR_UNSUPPORTED = -3


def _cdiv(a, b):
    return -(-a // b)


def scale_numel(rows, cols):
    """Bytes of the blocked scale buffer of a [rows, cols] operand (scripts/mxfp8.py:83-84)."""
    return _cdiv(rows, 128) * (cols // 128) * 512


def _check_bf16_2d(x2d, what):
    R, K = x2d.shape
    assert x2d.dtype == torch.bfloat16 and x2d.is_contiguous() and K % 128 == 0, (x2d.dtype, x2d.shape)
    if not x2d.is_cuda:
        raise RuntimeError(f"{what}: the MXFP8 kernels run on CUDA tensors only (got {x2d.device})")
    return R, K


def mx_quant(x2d):
    """[R, K] bf16 contiguous (K % 128 == 0) -> (fp8 e4m3 [R, K], e8m0 scales flat, cuBLAS blocked layout)."""
    R, K = _check_bf16_2d(x2d, "mx_quant")
    q = torch.empty((R, K), dtype=F8, device=x2d.device)
    s = torch.empty(scale_numel(R, K), dtype=torch.uint8, device=x2d.device)
    if R:
        _nx.call("mxm_quant_rows", _nx.ptr(x2d), R, K, K, _nx.ptr(q), K, _nx.ptr(s), _nx.stream_of(x2d))
    return q, s.view(E8)


def quant_ref(x2d):
    """Weight quantizer (scripts/mxfp8.py:40-43): row-wise, RCEIL scales, blocked layout."""
    x2d = x2d.contiguous()
    if x2d.dtype != torch.bfloat16:
        x2d = x2d.to(torch.bfloat16)
    return mx_quant(x2d)


def mx_quant_t(x2d):
    """Column-wise quantization: ``quant_ref(x2d.t().contiguous())`` without materializing the transpose.

    x2d [R, K] bf16, R % 128 == 0 -> (fp8 [K, R], scales blocked for [K, R]).
    """
    R, K = _check_bf16_2d(x2d, "mx_quant_t")
    assert R % 128 == 0, R
    qt = torch.empty((K, R), dtype=F8, device=x2d.device)
    st = torch.empty(scale_numel(K, R), dtype=torch.uint8, device=x2d.device)
    _nx.call("mxm_quant_cols", _nx.ptr(x2d), R, K, K, _nx.ptr(qt), _nx.ptr(st), _nx.stream_of(x2d))
    return qt, st.view(E8)


def mx_quant_pair(x2d):
    """Both orientations from one read: (q [R, K], s, qt [K, R], st).  R % 128 == 0."""
    R, K = _check_bf16_2d(x2d, "mx_quant_pair")
    assert R % 128 == 0, R
    dev = x2d.device
    q = torch.empty((R, K), dtype=F8, device=dev)
    s = torch.empty(scale_numel(R, K), dtype=torch.uint8, device=dev)
    qt = torch.empty((K, R), dtype=F8, device=dev)
    st = torch.empty(scale_numel(K, R), dtype=torch.uint8, device=dev)
    _nx.call("mxm_quant_both", _nx.ptr(x2d), R, K, K, _nx.ptr(q), _nx.ptr(s), _nx.ptr(qt), _nx.ptr(st),
             _nx.stream_of(x2d))
    return q, s.view(E8), qt, st.view(E8)


def mx_mm(a, b, scale_a, scale_b, out=None):
    """MXFP8 GEMM with ``torch._scaled_mm``'s convention: a [M, K] fp8 (row-major), b [K, N] fp8 given
    as the ``.t()`` of a row-major [N, K] matrix, scales blocked; returns bf16 [M, N]."""
    M, K = a.shape
    K2, N = b.shape
    assert K == K2 and a.dtype == F8 and b.dtype == F8, (a.shape, b.shape, a.dtype, b.dtype)
    bt = b.t()
    assert a.stride(1) == 1 and bt.stride(1) == 1, "operands must be K-contiguous"
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    _nx.call("mxm_gemm", _nx.ptr(a), a.stride(0), _nx.ptr(scale_a), _nx.ptr(bt), bt.stride(0), _nx.ptr(scale_b),
             M, N, K, _nx.ptr(out), out.stride(0), _nx.stream_of(a))
    return out


LORA_RANKS = (16, 32, 64)   # ranks the skinny kernels and the in-GEMM LoRA term take


def mx_mm_lora_ok(L, Rm):
    """Whether mx_mm_lora takes this LoRA term (rank in LORA_RANKS, bf16, 16-byte rows)."""
    return (L.shape[1] in LORA_RANKS and L.dtype == Rm.dtype == torch.bfloat16 and L.stride(1) == 1
            and L.stride(0) % 8 == 0 and L.data_ptr() % 16 == 0 and Rm.is_contiguous())


def mx_mm_lora(a, b, scale_a, scale_b, L, Rm):
    """bf16(mx_mm(a, b, ...) + L @ Rm^T): the MX GEMM with the rank-r LoRA term accumulated on the tensor
    core (Rm [N, r] bf16 contiguous already carries the LoRA scaling)."""
    M, K = a.shape
    N = b.shape[1]
    bt = b.t()
    kr = L.shape[1]
    assert Rm.is_contiguous() and Rm.shape == (N, kr) and L.stride(1) == 1
    out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    _nx.call("mxm_gemm_lora", _nx.ptr(a), a.stride(0), _nx.ptr(scale_a), _nx.ptr(bt), bt.stride(0), _nx.ptr(scale_b),
             M, N, K, _nx.ptr(L), L.stride(0), _nx.ptr(Rm), kr, _nx.ptr(out), out.stride(0), _nx.stream_of(a))
    return out


# ---------------------------------------------------------------------------------------------- LoRA backward
def lora_bwd_ok(dy, xa=None, B=None):
    """Whether lora_bwd's kernels take this branch: rank in LORA_RANKS and 16-byte aligned rows."""
    if dy.stride(0) % 8 or dy.data_ptr() % 16:
        return False
    if xa is None:
        return True
    return (xa.shape[1] in LORA_RANKS and xa.stride(1) == 1 and xa.stride(0) % 8 == 0 and xa.data_ptr() % 16 == 0
            and B.data_ptr() % 16 == 0)


def _branch(dy, xa, Bt, scale, dxa_out, dB):
    """One mxm_group_branch record (see include/mxmlp.h)."""
    b = _nx.GroupBranch()
    b.dy, b.ldy, b.N = dy.data_ptr(), dy.stride(0), dy.shape[1]
    if xa is not None:
        b.xa, b.ldxa, b.Bt, b.r, b.scale = xa.data_ptr(), xa.stride(0), Bt.data_ptr(), xa.shape[1], float(scale)
        b.dxa_out, b.ld_dxa, b.dB_out = dxa_out.data_ptr(), dxa_out.stride(0), dB.data_ptr()
    return b


def group_lora_bwd(T, branches, q=None, s=None, device=None):
    """The one-read backward of a group of MX linears in one native call (mxm_group_lora_bwd).  branches:
    (dy [T, N] bf16, xa [T, r] or None, B^T [r, N] bf16 contiguous or None, scale, dxa_out [T, r] or None,
    dB_out [N, r] fp32 or None) in the order of the group's K-concatenated dx operand q / s (None: no dx)."""
    recs = (_nx.GroupBranch * len(branches))(*[_branch(*br) for br in branches])
    need = 0
    for dy, xa, _, _, _, _ in branches:
        if xa is not None:
            need = max(need, _nx.coldot_chunks(T, dy.shape[1])[1] * dy.shape[1] * xa.shape[1])
    part = torch.empty(max(need, 1), dtype=torch.float32, device=device or branches[0][0].device)
    _nx.call("mxm_group_lora_bwd", T, len(branches), recs, _nx.ptr(q), q.stride(0) if q is not None else 0,
             _nx.ptr(s), q.shape[1] if q is not None else 0, _nx.ptr(part), part.numel() * 4,
             _nx.stream_of(branches[0][0]))


def lora_bwd(dy, xa=None, B=None, scale=1.0, q=None, s=None, col_tile_off=0, dxa_out=None):
    """One read of dy [T, N] bf16 (rows contiguous) for a LoRA branch over an MX base weight
    (scripts/mxfp8.py:219-263): with q / s, dy's row-wise MXFP8 goes into columns col_tile_off*128 .. of the
    K-concatenated q [T, sum N] (scales in q's blocked layout, byte-identical to mx_quant(dy)); with a
    LoRA branch (xa [T, r] = its columns of x S^T, B [N, r] bf16 contiguous) scale * dy @ B is written,
    rounded once to bf16, into dxa_out [T, r] and dB = scale * dy^T @ xa is returned in fp32.  A branch
    the kernels do not take (lora_bwd_ok) raises MXError(MXM_ERR_UNSUPPORTED)."""
    T, N = dy.shape
    assert dy.dtype == torch.bfloat16 and dy.stride(1) == 1 and N % 128 == 0, (dy.dtype, dy.shape, dy.stride())
    has_lora, do_q = xa is not None, q is not None
    if not (has_lora or do_q):
        return None
    if do_q:
        assert q.shape[0] == T and q.shape[1] % 128 == 0 and q.stride(1) == 1, (q.shape, q.stride())
        assert s.numel() == scale_numel(T, q.shape[1]), (s.numel(), T, q.shape)
    if not lora_bwd_ok(dy, xa, B):
        raise _nx.MXError("lora_bwd", MXM_ERR_UNSUPPORTED,
                          f"rank {None if xa is None else xa.shape[1]} or layout not taken by the kernels")
    if not has_lora:
        _nx.call("mxm_quant_rows_into", _nx.ptr(dy), T, N, dy.stride(0), _nx.ptr(q), q.stride(0), _nx.ptr(s),
                 q.shape[1], col_tile_off, _nx.stream_of(dy))
        return None
    R = xa.shape[1]
    assert B.is_contiguous() and B.shape == (N, R) and B.dtype == torch.bfloat16
    assert dxa_out.shape == (T, R) and dxa_out.stride(1) == 1
    Bt = B.t().contiguous()                                            # [r, N]: rows of the rowdot operand
    rpc, nch = _nx.coldot_chunks(T, N)
    part = torch.empty((nch, N, R), dtype=torch.float32, device=dy.device)
    dB = torch.empty((N, R), dtype=torch.float32, device=dy.device)
    _nx.call("mxm_lora_bwd", _nx.ptr(dy), dy.stride(0), T, N, _nx.ptr(xa), xa.stride(0), _nx.ptr(Bt), R,
             float(scale), _nx.ptr(q) if do_q else None, q.stride(0) if do_q else 0, _nx.ptr(s) if do_q else None,
             q.shape[1] if do_q else 0, col_tile_off, _nx.ptr(dxa_out), dxa_out.stride(0), _nx.ptr(dB),
             _nx.ptr(part), rpc, nch, _nx.stream_of(dy))
    return dB


def res_lora_ok(x, y, xa, B):
    """Whether res_lora's kernel takes these operands."""
    return (xa.shape[1] in LORA_RANKS and xa.stride(1) == 1 and xa.stride(0) % 2 == 0 and x.is_contiguous()
            and y.is_contiguous() and B.is_contiguous() and x.shape[-1] % 128 == 0
            and x.dtype == y.dtype == B.dtype == xa.dtype == torch.bfloat16 and x.numel() < 2**31)


def res_lora(x, y, xa, B, scale):
    """x + (y + scale * xa @ B^T) with the reference's two bf16 roundings (addmm, then the residual add), for
    x, y [T, N] bf16 contiguous, xa [T, r] (any row stride), B [N, r] contiguous -- scripts/mxfp8.py:285-296.
    Operands the kernel does not take (res_lora_ok) raise MXError(MXM_ERR_UNSUPPORTED)."""
    T, N = x.shape
    if not res_lora_ok(x, y, xa, B):
        raise _nx.MXError("res_lora", MXM_ERR_UNSUPPORTED, "rank, dtype or layout not taken by the kernel")
    out = torch.empty_like(x)
    _nx.call("mxm_res_lora", _nx.ptr(x), _nx.ptr(y), _nx.ptr(xa), xa.stride(0), _nx.ptr(B), T, N, xa.shape[1],
             float(scale), _nx.ptr(out), _nx.stream_of(x))
    return out


# ---------------------------------------------------------------------------------------------- weight layouts
# What enable_mxfp8 attaches to a frozen base linear.  The names are shared with fused_linear and
# fused_mlp, and the reference's caller tests `_mx_gu` on gate_proj (scripts/shared_prefix.py:189):
#   _mx_w, _mx_ws    W [N, K] codes quantized along K + scales (forward: x W^T)
#   _mx_wt, _mx_wts  W^T [K, N] codes quantized along N + scales (backward: dy W); single linears only
#   _mx_cat          (ConcatWT, position) for a member of a concatenated-W^T group
#   _mx_gu           (GateUp, 0 for gate / 1 for up) for the paired projections of one MLP
#   _mx_fbwd         whether fused_linear may run the one-read grouped backward for it
#   _bf16_cpu        the bf16 weight, parked in host memory while MXFP8 is on
_ATTRS = ("_mx_w", "_mx_ws", "_mx_wt", "_mx_wts", "_mx_cat", "_mx_gu", "_mx_fbwd", "_bf16_cpu", "forward")
_LINEAR_ROLES = frozenset({"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj",
                           "in_proj_qkv", "in_proj_z", "out_proj"})
# linears that share one input and whose dx is one GEMM against their concatenated W^T (fused_linear)
WT_GROUPS = (("in_proj_qkv", "in_proj_z"), ("q_proj", "k_proj", "v_proj"))
_CATS = WT_GROUPS
FUSED_BWD = {"in_proj_qkv", "in_proj_z", "q_proj", "k_proj", "v_proj", "o_proj", "out_proj"}
FUSE_GU = os.environ.get("MXFP8_FUSE_GU", "1") != "0"


def _blocked_cols(st, rows, cols, c0, c1):
    """Scales of columns [c0, c1) (multiples of 128) of a [rows, cols] operand in the blocked layout: per
    128-row block, the 512-byte tiles of those columns, gathered into a contiguous buffer."""
    t = st.view(torch.uint8).view(_cdiv(rows, 128), cols // 128, 512)
    return t[:, c0 // 128:c1 // 128].contiguous().view(-1).view(E8)


class GateUp:
    """The gate and up projections of one MLP as ONE matrix W_gu = [W_gate; W_up] [2N, K], quantized in both
    orientations (scripts/mxfp8.py:472-484): w / ws along K for the gate|up GEMM, wt / wts = W_gu^T [K, 2N]
    along 2N for dx.  A 32-block never straddles the gate/up boundary (N % 128 == 0), so every half is
    byte-identical to quantizing that projection alone: the first half of ws belongs to gate.  ``n`` = N."""

    def __init__(self, w_gate, w_up):
        self.n = w_gate.shape[0]
        both = torch.cat([w_gate, w_up]).to(torch.bfloat16).contiguous()
        self.w, self.ws, self.wt, self.wts = mx_quant_pair(both)
        self.half_t = [None, None]

    def rows(self, i):
        """(codes [N, K], scales) of projection i (0 gate, 1 up) for x W_i^T: views into w / ws."""
        ns = self.ws.numel() // 2
        return self.w[i * self.n:(i + 1) * self.n], self.ws[i * ns:(i + 1) * ns]

    def half(self, i):
        """(W_i^T codes [K, N] as a column range of wt, its scales gathered once) for dy W_i."""
        if self.half_t[i] is None:
            k = self.wt.shape[0]
            self.half_t[i] = (self.wt[:, i * self.n:(i + 1) * self.n],
                              _blocked_cols(self.wts, k, 2 * self.n, i * self.n, (i + 1) * self.n))
        return self.half_t[i]


class ConcatWT:
    """W^T of linears that share one input, concatenated along N and quantized once [K, sum N]
    (scripts/mxfp8.py:363-395): the whole group's dx is one GEMM against it, and a run of consecutive members
    is a column range (scales gathered on first use and kept)."""

    def __init__(self, lins):
        w = torch.cat([lin.weight.data for lin in lins], 0).to(torch.bfloat16).contiguous()
        self.qt, self.st = mx_quant_t(w)
        del w
        edges = [0]
        for lin in lins:
            edges.append(edges[-1] + lin.weight.shape[0])
        self.edges = edges
        self.n = len(lins)
        self._spans = {}

    def span(self, a, b):
        """(mat2 [N_a + .. + N_{b-1}, K] column-major view, scales) of members a .. b-1."""
        c0, c1 = self.edges[a], self.edges[b]
        mat2 = self.qt[:, c0:c1].t()
        if a == 0 and b == self.n:
            return mat2, self.st
        if (a, b) not in self._spans:
            self._spans[(a, b)] = _blocked_cols(self.st, self.qt.shape[0], self.qt.shape[1], c0, c1)
        return mat2, self._spans[(a, b)]

    range = span


def is_mx(lin):
    return getattr(lin, "_mx_w", None) is not None


def mx_wt(lin):
    """(fp8 W^T [K, N], scales) for dx = dy @ W (scripts/mxfp8.py:402-415)."""
    pair = lin.__dict__.get("_mx_gu")
    if pair is not None:
        return pair[0].half(pair[1])
    mat2, s = wt_of(lin)
    return mat2.t(), s


def wt_of(lin):
    """(mat2, scales) of dy @ W for one linear; mat2 = W^T codes as a [N, K] column-major view
    (scripts/mxfp8.py:418-426)."""
    d = lin.__dict__
    if "_mx_cat" in d:
        cat, k = d["_mx_cat"]
        return cat.span(k, k + 1)
    if "_mx_gu" in d:
        hold, i = d["_mx_gu"]
        wt, s = hold.half(i)
        return wt.t(), s
    return lin._mx_wt.t(), lin._mx_wts


def group_wt(lins):
    """(mat2 [sum N, K], scales) for dx of consecutive linears of one concatenated group, or None
    (scripts/mxfp8.py:429-439)."""
    tags = [lin.__dict__.get("_mx_cat") for lin in lins]
    if tags[0] is None:
        return wt_of(lins[0]) if len(lins) == 1 else None
    cat, k0 = tags[0]
    if any(t is None or t[0] is not cat or t[1] != k0 + j for j, t in enumerate(tags)):
        return None
    return cat.span(k0, k0 + len(lins))


# ---- planning: which layout each frozen linear gets
def _frozen_linears(model):
    """(parent path, role, linear) of every frozen, bias-free base linear of the decoder blocks whose role is
    one of _LINEAR_ROLES (a PEFT wrapper's base_layer counts under the wrapper's name) -- the linears the
    reference converts (scripts/mxfp8.py:347-356)."""
    for name, mod in model.named_modules():
        if not isinstance(mod, torch.nn.Linear) or mod.weight.requires_grad or ".layers." not in name:
            continue
        stem = name[:-len(".base_layer")] if name.endswith(".base_layer") else name
        parent, _, role = stem.rpartition(".")
        if role in _LINEAR_ROLES:
            yield parent, role, mod


def _plan(model):
    """The layouts enable_mxfp8 builds, as (kind, linears, one_read) steps: "pair" (gate, up) of one MLP,
    "cat" for a W^T group, then "single" (with its own W^T) / "member" (forward codes only: its W^T lives
    in the group) for every linear.  Groups are found per parent module."""
    by_parent = {}
    for parent, role, lin in _frozen_linears(model):
        assert lin.bias is None
        w = lin.weight
        assert w.is_cuda and w.shape[0] % 128 == 0 and w.shape[1] % 128 == 0, (parent, role, tuple(w.shape))
        by_parent.setdefault(parent, []).append((role, lin))
    steps, placed = [], {}
    for parent in by_parent:
        roles = dict(by_parent[parent])
        for group in WT_GROUPS:
            if all(r in roles for r in group):
                steps.append(("cat", tuple(roles[r] for r in group)))
                placed.update({id(roles[r]): "member" for r in group})
        gate, up = roles.get("gate_proj"), roles.get("up_proj")
        if FUSE_GU and gate is not None and up is not None and gate.weight.shape == up.weight.shape:
            steps.append(("pair", (gate, up)))
            placed.update({id(gate): "paired", id(up): "paired"})
    for parent in by_parent:
        for role, lin in by_parent[parent]:
            steps.append((placed.get(id(lin), "single"), (lin,), role in FUSED_BWD))
    return steps


def _build(step):
    kind, lins = step[0], step[1]
    if kind == "cat":
        cat = ConcatWT(lins)
        for k, lin in enumerate(lins):
            lin._mx_cat = (cat, k)
    elif kind == "pair":
        hold = GateUp(lins[0].weight.data, lins[1].weight.data)
        for i, lin in enumerate(lins):
            lin._mx_w, lin._mx_ws = hold.rows(i)
            lin._mx_gu = (hold, i)
    else:
        (lin,) = lins
        w = lin.weight.data
        if kind == "single":
            lin._mx_w, lin._mx_ws, lin._mx_wt, lin._mx_wts = mx_quant_pair(w.to(torch.bfloat16).contiguous())
        elif kind == "member":
            lin._mx_w, lin._mx_ws = quant_ref(w)
        lin._mx_fbwd = step[2]
        lin._bf16_cpu = w.to("cpu", copy=True)
        lin.weight.data = torch.empty((0,), dtype=w.dtype, device=w.device)   # dtype / device stay readable
        lin.forward = types.MethodType(_mx_linear_forward, lin)


def enable_mxfp8(model):
    """Quantize every frozen base linear of the decoder blocks once, in both orientations; pair gate|up of
    each MLP into one W_gu = [W_gate; W_up] (scripts/mxfp8.py:452-498).  Returns the number of linears."""
    steps = _plan(model)
    for st in steps:               # groups and pairs read the bf16 weights: before any weight is parked
        if st[0] in ("cat", "pair"):
            _build(st)
    per_lin = [st for st in steps if st[0] not in ("cat", "pair")]
    for st in per_lin:
        _build(st)
    torch.cuda.empty_cache()
    n_cat = sum(len(st[1]) for st in steps if st[0] == "cat")
    n_pair = sum(1 for st in steps if st[0] == "pair")
    print(f"MXFP8: {len(per_lin)} frozen linears on MXFP8 GEMMs (bf16 weights moved to host memory;"
          f" {n_cat} in concatenated W^T groups, {n_pair} gate/up pairs)", flush=True)
    return len(per_lin)


def disable_mxfp8(model):
    """Undo enable_mxfp8: bf16 weights back on the device, every attribute it added removed
    (scripts/mxfp8.py:501-509)."""
    for _, _, lin in _frozen_linears(model):
        d = lin.__dict__
        if "_bf16_cpu" not in d:
            continue
        lin.weight.data = d["_bf16_cpu"].to(lin.weight.device)
        for a in _ATTRS:
            d.pop(a, None)
    _ACT.clear()
    torch.cuda.empty_cache()


# ---------------------------------------------------------------------------------------------- MX linears
class _ActQuantCache:
    """The MXFP8 of the last linear input quantized (scripts/mxfp8.py:299-312): q/k/v, qkv/z and gate/up
    receive the same tensor, which is then quantized once.  A weak reference plus the tensor's version
    counter identify it, so neither a freed tensor whose memory was reused nor an in-place update hits."""

    def __init__(self):
        self.clear()

    def clear(self):
        self.ref, self.version, self.qs = None, -1, None

    def get(self, x):
        if self.ref is not None and self.ref() is x and self.version == x._version:
            STATS["reuse"] += 1
            return self.qs
        x2 = x.reshape(-1, x.shape[-1])
        if x2.dtype != torch.bfloat16 or not x2.is_contiguous():
            x2 = x2.to(torch.bfloat16).contiguous()
        self.qs = mx_quant(x2)
        STATS["quant"] += 1
        self.ref, self.version = weakref.ref(x), x._version
        return self.qs


_ACT = _ActQuantCache()


class _MXMatmul(torch.autograd.Function):
    """y = x W^T from the input's MX codes; dx = MXFP8(dy) W (scripts/mxfp8.py:315-333).  The base weight is
    frozen: no weight gradient."""

    @staticmethod
    def forward(ctx, x, q, s, lin):
        ctx.lin = lin
        y = mx_mm(q, lin._mx_w.t(), s, lin._mx_ws)
        return y.view(*x.shape[:-1], y.shape[-1])

    @staticmethod
    def backward(ctx, dy):
        d2 = dy.reshape(-1, dy.shape[-1])
        if d2.dtype != torch.bfloat16 or not d2.is_contiguous():
            d2 = d2.to(torch.bfloat16).contiguous()
        qd, sd = mx_quant(d2)
        STATS["quant"] += 1
        mat2, ws = wt_of(ctx.lin)
        dx = mx_mm(qd, mat2, sd, ws)
        return dx.view(*dy.shape[:-1], dx.shape[-1]), None, None, None


@torch.compiler.disable
def _mx_linear_forward(self, x):
    """forward of a converted base linear (kept out of torch.compile regions, as the reference does)."""
    q, s = _ACT.get(x)
    return _MXMatmul.apply(x, q, s, self)
