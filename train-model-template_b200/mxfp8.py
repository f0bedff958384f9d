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
  (``b`` is the ``.t()`` view of a [N, K] code matrix), on the tcgen05 block-scaled MMA.
* ``enable_mxfp8`` / ``disable_mxfp8`` / ``is_mx`` / ``mx_wt`` / ``wt_of`` / ``group_wt`` -- the frozen
  weight layout builder (scripts/mxfp8.py:398-509), including the shared gate|up pair that
  ``fused_mlp`` consumes.
* ``lora_bwd`` / ``res_lora`` -- the LoRA backward of an MX linear from one read of dy (MXFP8 of dy into a
  K-concatenated buffer + d(xa) + dB) and the residual add with the LoRA term, used by ``fused_linear``
  (scripts/mxfp8.py:88-296).
"""
import ctypes
import os
import types
import weakref

import torch

import _mxlib as _nx

F8, E8 = torch.float8_e4m3fn, torch.float8_e8m0fnu
STATS = {"quant": 0, "reuse": 0}


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


# ---------------------------------------------------------------------------------------------- LoRA backward
_rowdot_ns = (16, 32, 64)


def _native_lora_ok(dy, xa, B, R):
    return (R in _rowdot_ns and dy.stride(0) % 8 == 0 and xa.stride(0) % 8 == 0 and xa.data_ptr() % 16 == 0
            and dy.data_ptr() % 16 == 0 and B.data_ptr() % 16 == 0)


def lora_bwd(dy, xa=None, B=None, scale=1.0, q=None, s=None, col_tile_off=0, dxa_out=None):
    """One read of dy [T, N] bf16 (rows contiguous) for a LoRA branch over an MX base weight
    (scripts/mxfp8.py:219-263): with q / s, dy's row-wise MXFP8 goes into columns col_tile_off*128 .. of the
    K-concatenated q [T, sum N] (scales in q's blocked layout, byte-identical to mx_quant(dy)); with a
    LoRA branch (xa [T, r] = its columns of x S^T, B [N, r] bf16 contiguous) scale * dy @ B is written,
    rounded once to bf16, into dxa_out [T, r] and dB = scale * dy^T @ xa is returned in fp32."""
    T, N = dy.shape
    assert dy.dtype == torch.bfloat16 and dy.stride(1) == 1 and N % 128 == 0, (dy.dtype, dy.shape, dy.stride())
    has_lora, do_q = xa is not None, q is not None
    if not (has_lora or do_q):
        return None
    assert T * max(dy.stride(0), q.shape[1] if do_q else 0) < 2**31
    if do_q:
        assert q.shape[0] == T and q.shape[1] % 128 == 0 and q.stride(1) == 1, (q.shape, q.stride())
        assert s.numel() == scale_numel(T, q.shape[1]), (s.numel(), T, q.shape)
    if not has_lora:
        _nx.call("mxm_quant_rows_into", _nx.ptr(dy), T, N, dy.stride(0), _nx.ptr(q), q.stride(0), _nx.ptr(s),
                 q.shape[1], col_tile_off, _nx.stream_of(dy))
        return None
    R = xa.shape[1]
    assert xa.stride(1) == 1 and B.is_contiguous() and B.shape == (N, R) and B.dtype == torch.bfloat16
    assert dxa_out.shape == (T, R) and dxa_out.stride(1) == 1
    if not _native_lora_ok(dy, xa, B, R):
        # ranks / layouts the kernels do not take: the same products with torch GEMMs (fp32 accumulate)
        if do_q:
            lora_bwd(dy, q=q, s=s, col_tile_off=col_tile_off)
        dxa_out.copy_(((dy.float() @ B.float()) * scale).to(dxa_out.dtype))
        return (dy.t().float() @ xa.float()) * scale
    Bt = B.t().contiguous()                                            # [r, N]: rows of the rowdot operand
    rpc, nch = ctypes.c_int(0), ctypes.c_int(0)
    _nx.call("mxm_coldot_chunks", T, N, _nx.ctypes_ref(rpc), _nx.ctypes_ref(nch))
    part = torch.empty((nch.value, N, R), dtype=torch.float32, device=dy.device)
    dB = torch.empty((N, R), dtype=torch.float32, device=dy.device)
    _nx.call("mxm_lora_bwd", _nx.ptr(dy), dy.stride(0), T, N, _nx.ptr(xa), xa.stride(0), _nx.ptr(Bt), R,
             float(scale), _nx.ptr(q) if do_q else None, q.stride(0) if do_q else 0, _nx.ptr(s) if do_q else None,
             q.shape[1] if do_q else 0, col_tile_off, _nx.ptr(dxa_out), dxa_out.stride(0), _nx.ptr(dB),
             _nx.ptr(part), rpc.value, nch.value, _nx.stream_of(dy))
    return dB


def res_lora(x, y, xa, B, scale):
    """x + (y + scale * xa @ B^T) with the reference's two bf16 roundings (addmm, then the residual add), for
    x, y [T, N] bf16 contiguous, xa [T, r] (any row stride), B [N, r] contiguous -- scripts/mxfp8.py:285-296."""
    T, N = x.shape
    assert T * N < 2**31 and N % 128 == 0
    out = torch.empty_like(x)
    R = xa.shape[1]
    if (R in _rowdot_ns and xa.stride(1) == 1 and xa.stride(0) % 2 == 0 and x.is_contiguous() and y.is_contiguous()
            and B.is_contiguous() and x.dtype == y.dtype == B.dtype == xa.dtype == torch.bfloat16):
        _nx.call("mxm_res_lora", _nx.ptr(x), _nx.ptr(y), _nx.ptr(xa), xa.stride(0), _nx.ptr(B), T, N, R,
                 float(scale), _nx.ptr(out), _nx.stream_of(x))
        return out
    t = (y.float() + scale * (xa.float() @ B.float().t())).to(torch.bfloat16)
    return out.copy_((x.float() + t.float()).to(x.dtype))


# ---------------------------------------------------------------------------------------------- MX linears
_last = [None, 0, None, None]  # (weakref of the last quantized input, its _version, q, s)


def _quant_act(x):
    """Quantize a linear's input, reusing the result when the same tensor is quantized again
    (q/k/v, qkv/z and gate/up share one input) -- scripts/mxfp8.py:299-312."""
    if _last[0] is not None and _last[0]() is x and _last[1] == x._version:
        STATS["reuse"] += 1
        return _last[2], _last[3]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.bfloat16 or not x2.is_contiguous():
        x2 = x2.to(torch.bfloat16).contiguous()
    q, s = mx_quant(x2)
    STATS["quant"] += 1
    _last[:] = [weakref.ref(x), x._version, q, s]
    return q, s


class _MXLinear(torch.autograd.Function):
    """y = x @ W^T on MX codes; backward dx = dy @ W (scripts/mxfp8.py:315-333)."""

    @staticmethod
    def forward(ctx, x, q, s, lin):
        out = mx_mm(q, lin._mx_w.t(), s, lin._mx_ws)
        ctx.lin = lin
        return out.view(*x.shape[:-1], out.shape[-1])

    @staticmethod
    def backward(ctx, dy):
        lin = ctx.lin
        n = dy.shape[-1]
        dy2 = dy.reshape(-1, n)
        if dy2.dtype != torch.bfloat16 or not dy2.is_contiguous():
            dy2 = dy2.to(torch.bfloat16).contiguous()
        q, s = mx_quant(dy2)
        STATS["quant"] += 1
        wt, wts = wt_of(lin)
        dx = mx_mm(q, wt, s, wts)
        return dx.view(*dy.shape[:-1], dx.shape[-1]), None, None, None


@torch.compiler.disable
def _forward(self, x):
    q, s = _quant_act(x)
    return _MXLinear.apply(x, q, s, self)


_NAMES = {"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "in_proj_qkv", "in_proj_z",
          "out_proj"}


def _base_linears(model):
    """Frozen base linears of the decoder blocks (scripts/mxfp8.py:347-356)."""
    for name, m in model.named_modules():
        if not isinstance(m, torch.nn.Linear) or m.weight.requires_grad or ".layers." not in name:
            continue
        parts = name.split(".")
        leaf = parts[-2] if parts[-1] == "base_layer" else parts[-1]
        if leaf in _NAMES:
            yield name, m


_CATS = (("in_proj_qkv", "in_proj_z"), ("q_proj", "k_proj", "v_proj"))
FUSED_BWD = {"in_proj_qkv", "in_proj_z", "q_proj", "k_proj", "v_proj", "o_proj", "out_proj"}


class _Cat:
    """Concatenated W^T [K, sum N] codes + scales of a group of linears sharing one input
    (scripts/mxfp8.py:369-395)."""

    def __init__(self, lins):
        w = torch.cat([lin.weight.data for lin in lins], 0).to(torch.bfloat16)
        self.qt, self.st = mx_quant_t(w.contiguous())
        del w
        self.offs = [0]
        for lin in lins:
            self.offs.append(self.offs[-1] + lin.weight.shape[0])
        self.n = len(lins)
        self._sub = {}

    def range(self, a, b):
        c0, c1 = self.offs[a], self.offs[b]
        mat2 = self.qt[:, c0:c1].t()
        if (a, b) == (0, self.n):
            return mat2, self.st
        sc = self._sub.get((a, b))
        if sc is None:
            K, ntot = self.qt.shape
            blk = self.st.view(torch.uint8).view(_cdiv(K, 128), ntot // 128, 512)
            sc = self._sub[(a, b)] = blk[:, c0 // 128:c1 // 128].contiguous().view(-1).view(E8)
        return mat2, sc


def is_mx(lin):
    return getattr(lin, "_mx_w", None) is not None


def mx_wt(lin):
    """(fp8 W^T [K, N], scales) for dx = dy @ W (scripts/mxfp8.py:402-415)."""
    gu = lin.__dict__.get("_mx_gu")
    if gu is None:
        m, s = wt_of(lin)
        return m.t(), s
    hold, i = gu
    if hold.half_t[i] is None:
        n, k = hold.n, hold.wt.shape[0]
        s3 = hold.wts.view(torch.uint8).view(k // 128, 2 * n // 128, 512)
        hold.half_t[i] = (hold.wt[:, i * n:(i + 1) * n],
                          s3[:, i * (n // 128):(i + 1) * (n // 128)].reshape(-1).view(E8))
    return hold.half_t[i]


def wt_of(lin):
    """(mat2, scales) of dy @ W for one linear; mat2 = W^T codes as a [N, K] column-major view
    (scripts/mxfp8.py:418-426)."""
    c = lin.__dict__.get("_mx_cat")
    if c is not None:
        return c[0].range(c[1], c[1] + 1)
    if "_mx_gu" in lin.__dict__:
        wt, s = mx_wt(lin)
        return wt.t(), s
    return lin._mx_wt.t(), lin._mx_wts


def group_wt(lins):
    """(mat2 [sum N, K], scales) for dx of consecutive linears of one concatenated group, or None
    (scripts/mxfp8.py:429-439)."""
    c = lins[0].__dict__.get("_mx_cat")
    if c is None:
        return wt_of(lins[0]) if len(lins) == 1 else None
    cat, k = c
    for d, lin in enumerate(lins):
        if lin.__dict__.get("_mx_cat") != (cat, k + d):
            return None
    return cat.range(k, k + len(lins))


def _leaf_parent(name):
    parts = name.split(".")
    if parts[-1] == "base_layer":
        return parts[-2], ".".join(parts[:-2])
    return parts[-1], ".".join(parts[:-1])


FUSE_GU = os.environ.get("MXFP8_FUSE_GU", "1") != "0"


def enable_mxfp8(model):
    """Quantize every frozen base linear of the decoder blocks once, in both orientations; pair
    gate|up of each MLP into one W_gu = [W_gate; W_up] (scripts/mxfp8.py:452-498)."""
    lins = list(_base_linears(model))
    fam = {}
    for name, lin in lins:
        assert lin.bias is None
        w = lin.weight.data
        assert w.is_cuda and w.shape[0] % 128 == 0 and w.shape[1] % 128 == 0, w.shape
        leaf, parent = _leaf_parent(name)
        fam.setdefault(parent, {})[leaf] = lin
    in_cat, paired = set(), set()
    for d in fam.values():
        for names in _CATS:
            if all(k in d for k in names):
                grp = [d[k] for k in names]
                cat = _Cat(grp)
                for k, lin in enumerate(grp):
                    lin._mx_cat = (cat, k)
                    in_cat.add(id(lin))
        gb, ub = d.get("gate_proj"), d.get("up_proj")
        if FUSE_GU and gb is not None and ub is not None and gb.weight.shape == ub.weight.shape:
            w = torch.cat([gb.weight.data, ub.weight.data]).to(torch.bfloat16).contiguous()   # [2N, K]
            n = gb.weight.shape[0]
            hold = types.SimpleNamespace(n=n, half_t=[None, None])
            hold.w, hold.ws, hold.wt, hold.wts = mx_quant_pair(w)
            del w
            ns = hold.ws.numel() // 2
            for i, lin in enumerate((gb, ub)):
                lin._mx_w, lin._mx_ws = hold.w[i * n:(i + 1) * n], hold.ws[i * ns:(i + 1) * ns]
                lin._mx_gu = (hold, i)
                paired.add(id(lin))
    for name, lin in lins:
        w = lin.weight.data
        if id(lin) not in paired:
            wb = w.to(torch.bfloat16).contiguous()
            if id(lin) not in in_cat:
                lin._mx_w, lin._mx_ws, lin._mx_wt, lin._mx_wts = mx_quant_pair(wb)
            else:
                lin._mx_w, lin._mx_ws = quant_ref(wb)
            del wb
        lin._mx_fbwd = _leaf_parent(name)[0] in FUSED_BWD
        lin._bf16_cpu = w.to("cpu", copy=True)
        lin.weight.data = torch.empty((0,), dtype=w.dtype, device=w.device)
        lin.forward = types.MethodType(_forward, lin)
    torch.cuda.empty_cache()
    print(f"MXFP8: {len(lins)} frozen linears on MXFP8 GEMMs (bf16 weights moved to host memory;"
          f" {len(in_cat)} in concatenated W^T groups, {len(paired) // 2} gate/up pairs)", flush=True)
    return len(lins)


def disable_mxfp8(model):
    """Undo enable_mxfp8: bf16 weights back on the device, patches removed (scripts/mxfp8.py:501-509)."""
    for _, lin in _base_linears(model):
        if hasattr(lin, "_bf16_cpu"):
            lin.weight.data = lin._bf16_cpu.to(lin.weight.device)
            for a in ("_mx_w", "_mx_ws", "_mx_wt", "_mx_wts", "_mx_cat", "_mx_gu", "_mx_fbwd", "_bf16_cpu", "forward"):
                if a in lin.__dict__:
                    delattr(lin, a)
    _last[:] = [None, 0, None, None]
    torch.cuda.empty_cache()
