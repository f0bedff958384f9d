"""tcgen05 MXFP8 GEMM vs the oracle (dequantize + fp32 matmul) and vs torch._scaled_mm (cuBLASLt)."""
import numpy as np
import pytest
import torch

from oracle import mx_oracle as O

pytestmark = pytest.mark.gpu
TOL = 5e-3   # relative Frobenius error, the parity bar for outputs


def _rel(a, b):
    a = a.double()
    b = b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (200, 512, 384), (1, 256, 256), (77, 768, 1024),
                                   (1000, 1024, 512), (2049, 256, 2048), (512, 12288, 2048)])
def test_gemm_vs_oracle(M, N, K):
    import mxfp8
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    qa, sa = mxfp8.mx_quant(a.cuda())
    qb, sb = mxfp8.mx_quant(b.cuda())
    d = mxfp8.mx_mm(qa, qb.t(), sa, sb)
    torch.cuda.synchronize()
    ref = O.mx_gemm(qa.view(torch.uint8).cpu().numpy(), sa.view(torch.uint8).cpu().numpy(),
                    qb.view(torch.uint8).cpu().numpy(), sb.view(torch.uint8).cpu().numpy(), M, N, K)
    err = _rel(d.float().cpu(), torch.from_numpy(ref))
    assert err < 2e-3, err
    import _mxlib
    assert _mxlib.device_error() == 0


@pytest.mark.parametrize("N", [2048, 6144])
def test_gemm_vs_cublaslt(N):
    import mxfp8
    M, K = 1024, 2048
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    b = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    qa, sa = mxfp8.mx_quant(a)
    qb, sb = mxfp8.mx_quant(b)
    d = mxfp8.mx_mm(qa, qb.t(), sa, sb)
    try:
        ref = torch._scaled_mm(qa, qb.t(), sa, sb, out_dtype=torch.bfloat16)
    except Exception as e:  # pragma: no cover - depends on the torch build
        pytest.skip(f"torch._scaled_mm MX path unavailable: {e}")
    assert _rel(d.float(), ref.float()) < 2e-3


def test_gemm_strided_operand_and_determinism():
    """B given as a column slice with row stride 2N (the gate / up halves of W_gu^T)."""
    import mxfp8
    M, N, K = 256, 512, 256
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = torch.randn(K, 2 * N, device="cuda").to(torch.bfloat16)   # [K, 2N] -> operand [N, K] column slices
    qa, sa = mxfp8.mx_quant(a)
    qw, sw = mxfp8.mx_quant(w.t().contiguous())        # [2N, K]
    full = mxfp8.mx_mm(qa, qw.t(), sa, sw)
    half = mxfp8.mx_mm(qa, qw[N:].t(), sa, sw.view(torch.uint8)[sw.numel() // 2:].view(torch.float8_e8m0fnu))
    assert torch.equal(full[:, N:], half)
    again = mxfp8.mx_mm(qa, qw.t(), sa, sw)
    assert torch.equal(full, again)


@pytest.mark.parametrize("M,N,K,kr", [(300, 512, 256, 16), (1000, 2048, 1024, 32), (129, 256, 384, 64)])
def test_gemm_lora_vs_oracle(M, N, K, kr):
    """D = bf16(dq(A) dq(B)^T + L Rm^T): the LoRA term accumulated by a bf16 tcgen05 MMA."""
    import fused_mlp
    import mxfp8
    g = torch.Generator().manual_seed(M + kr)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    L = (torch.randn(M, kr, generator=g) * 0.5).to(torch.bfloat16)
    Rm = (torch.randn(N, kr, generator=g) * 0.1).to(torch.bfloat16)
    qa, sa = mxfp8.mx_quant(a.cuda())
    qb, sb = mxfp8.mx_quant(b.cuda())
    d = fused_mlp.mx_mm_lora(qa, qb.t(), sa, sb, L.cuda(), Rm.cuda())
    torch.cuda.synchronize()
    A = O.mx_dequant(qa.view(torch.uint8).cpu().numpy(), sa.view(torch.uint8).cpu().numpy(), M, K)
    B = O.mx_dequant(qb.view(torch.uint8).cpu().numpy(), sb.view(torch.uint8).cpu().numpy(), N, K)
    ref = A @ B.T + L.float().numpy() @ Rm.float().numpy().T
    err = _rel(d.float().cpu(), torch.from_numpy(ref))
    assert err < 2e-3, err
